// Python bindings of the symmetric heap (CUDA IPC) and the NVLink peer-memory kernels.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <cstring>

namespace cb {
cudaError_t signal_peers(const uint64_t* peer_flag_ptrs, int world, int slot, uint32_t epoch, cudaStream_t s);
cudaError_t wait_flags(const uint32_t* flags, int world, uint32_t epoch, int* status, uint64_t limit_ns,
                       cudaStream_t s);
cudaError_t p2p_barrier(const uint64_t* peer_flag_ptrs, int world, int my_rank, uint32_t* epoch_ctr,
                        const uint32_t* my_flags, int* status, uint64_t limit_ns, cudaStream_t s);
cudaError_t p2p_gather_rows(const void* src, int n, int row_bytes, const uint64_t* dst_ptrs, int world, int row0,
                            cudaStream_t s);
cudaError_t p2p_scatter_partials(const void* part, int T, int D, const int* bounds_dev, int world, int my_rank,
                                 const uint64_t* slot_ptrs, int slot_rows, cudaStream_t s);
cudaError_t reduce_slots(const void* slots, int world, int slot_rows, int n, int D, void* out, cudaStream_t s);
cudaError_t p2p_a2a_heads(const void* src, const int* bounds_dev, int world, int my_rank, const uint64_t* dst_ptrs,
                          int C, int mode, int max_rows, cudaStream_t s);
cudaError_t moe_count(const int* ids, int Tk, int E, int world, int my_rank, const uint64_t* cnt_ptrs,
                      int* pair_rank, cudaStream_t s);
cudaError_t moe_layout(const int* cnt, int world, int E, int my_rank, int max_blocks, int align, int* my_off,
                       int* m_block_expert, int* num_blocks, cudaStream_t s);
cudaError_t moe_dispatch(const void* x, int T, int D, const int* ids, int k, int El, int my_rank,
                         const int* pair_rank, const uint64_t* recv_ptrs, const uint64_t* sf_ptrs,
                         const int* my_off, const uint64_t* rinfo_ptrs, int cap, int* pos_out, int* status,
                         cudaStream_t s);
cudaError_t moe_combine_slots(const void* slots, int T, int D, const int* pos, const float* w, int k, const void* add,
                              void* out, cudaStream_t s);
cudaError_t moe_combine_pull(const uint64_t* y_ptrs, int T, int D, const int* ids, const int* pos, const float* w,
                             int k, int El, const void* add, void* out, cudaStream_t s);
cudaError_t embed_peer(const uint64_t* table_ptrs, int per, int world, const int* ids, int T, int D, int hc,
                       void* X, float* sumsq, cudaStream_t s);
cudaError_t gemm_fp8_scatter(const void* A, const void* B, const uint32_t* sfa, const uint32_t* sfb, int M, int N,
                             int K, const uint64_t* scatter_ptrs, const int* bounds, int world, int my_rank,
                             int slot_rows, int* status, int num_sms, cudaStream_t s);
cudaError_t gemm_fp8_push(const void* A, const void* B, const uint32_t* sfa, const uint32_t* sfb, int M, int N, int K,
                          int Nb, const int* m_block_expert, const int* num_m_blocks_dev, int max_m_blocks,
                          const int* row_dst, const uint64_t* home_ptrs, int world, int* status, int num_sms,
                          cudaStream_t s);
}  // namespace cb

namespace {

#define CKP(expr)                                                                          \
  do {                                                                                     \
    cudaError_t _e = (expr);                                                               \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));             \
  } while (0)

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }
const uint64_t* u64(const torch::Tensor& t) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kLong && t.is_contiguous(), "pointer table: int64 CUDA tensor");
  return reinterpret_cast<const uint64_t*>(t.data_ptr());
}

// -- heap ------------------------------------------------------------------------------------------------------------
int64_t symm_malloc(int64_t nbytes) {
  void* p = nullptr;
  CKP(cudaMalloc(&p, size_t(nbytes)));
  CKP(cudaMemset(p, 0, size_t(nbytes)));
  return reinterpret_cast<int64_t>(p);
}
void symm_free(int64_t p) { CKP(cudaFree(reinterpret_cast<void*>(p))); }
pybind11::bytes symm_ipc_handle(int64_t p) {
  cudaIpcMemHandle_t h;
  CKP(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(p)));
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}
int64_t symm_ipc_open(pybind11::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  CKP(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}
void symm_ipc_close(int64_t p) { CKP(cudaIpcCloseMemHandle(reinterpret_cast<void*>(p))); }

// Non-owning tensor view of heap memory.
torch::Tensor tensor_from_ptr(int64_t p, std::vector<int64_t> shape, const std::string& dtype, int64_t device) {
  at::ScalarType st;
  if (dtype == "bfloat16") st = at::kBFloat16;
  else if (dtype == "float32") st = at::kFloat;
  else if (dtype == "int32") st = at::kInt;
  else if (dtype == "int64") st = at::kLong;
  else if (dtype == "uint8") st = at::kByte;
  else if (dtype == "float8_e4m3fn") st = at::kFloat8_e4m3fn;
  else if (dtype == "float16") st = at::kHalf;
  else TORCH_CHECK(false, "tensor_from_ptr: unsupported dtype ", dtype);
  auto opts = torch::TensorOptions().dtype(st).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(p), shape, opts);
}

// -- signals ---------------------------------------------------------------------------------------------------------
void signal_peers(torch::Tensor peer_flag_ptrs, int64_t slot, int64_t epoch) {
  CKP(cb::signal_peers(u64(peer_flag_ptrs), peer_flag_ptrs.numel(), slot, uint32_t(epoch), stream()));
}
void wait_flags(torch::Tensor flags, int64_t world, int64_t epoch, torch::Tensor status, int64_t limit_ns) {
  CKP(cb::wait_flags(reinterpret_cast<const uint32_t*>(flags.data_ptr()), world, uint32_t(epoch),
                     status.data_ptr<int>(), uint64_t(limit_ns), stream()));
}

void p2p_barrier(torch::Tensor peer_flag_ptrs, int64_t my_rank, torch::Tensor epoch_ctr, torch::Tensor my_flags,
                 torch::Tensor status, int64_t limit_ns) {
  CKP(cb::p2p_barrier(u64(peer_flag_ptrs), peer_flag_ptrs.numel(), my_rank,
                      reinterpret_cast<uint32_t*>(epoch_ctr.data_ptr()),
                      reinterpret_cast<const uint32_t*>(my_flags.data_ptr()), status.data_ptr<int>(),
                      uint64_t(limit_ns), stream()));
}

// -- data movement ---------------------------------------------------------------------------------------------------
void p2p_gather_rows(torch::Tensor src, torch::Tensor dst_ptrs, int64_t row0) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous());
  const int n = src.size(0);
  const int row_bytes = n ? int(src.numel() / n * src.element_size()) : 0;
  CKP(cb::p2p_gather_rows(src.data_ptr(), n, row_bytes, u64(dst_ptrs), dst_ptrs.numel(), row0, stream()));
}
void p2p_scatter_partials(torch::Tensor part, torch::Tensor bounds, int64_t my_rank, torch::Tensor slot_ptrs,
                          int64_t slot_rows) {
  TORCH_CHECK(part.is_cuda() && part.is_contiguous() && part.scalar_type() == at::kBFloat16);
  CKP(cb::p2p_scatter_partials(part.data_ptr(), part.size(0), part.size(1), bounds.data_ptr<int>(),
                               slot_ptrs.numel(), my_rank, u64(slot_ptrs), slot_rows, stream()));
}
void reduce_slots(torch::Tensor slots, int64_t world, int64_t slot_rows, int64_t n, torch::Tensor out) {
  CKP(cb::reduce_slots(slots.data_ptr(), world, slot_rows, n, out.size(1), out.data_ptr(), stream()));
}
void p2p_a2a_heads(torch::Tensor src, torch::Tensor bounds, int64_t my_rank, torch::Tensor dst_ptrs,
                   int64_t block_bytes, int64_t mode, int64_t max_rows) {
  TORCH_CHECK(src.is_cuda() && src.is_contiguous() && bounds.scalar_type() == at::kInt);
  CKP(cb::p2p_a2a_heads(src.data_ptr(), bounds.data_ptr<int>(), dst_ptrs.numel(), my_rank, u64(dst_ptrs),
                        block_bytes, mode, max_rows, stream()));
}
void moe_count(torch::Tensor ids, int64_t E, int64_t my_rank, torch::Tensor cnt_ptrs, torch::Tensor pair_rank) {
  TORCH_CHECK(ids.is_contiguous() && ids.scalar_type() == at::kInt);
  CKP(cb::moe_count(ids.data_ptr<int>(), ids.numel(), E, cnt_ptrs.numel(), my_rank, u64(cnt_ptrs),
                    pair_rank.data_ptr<int>(), stream()));
}
void moe_layout(torch::Tensor cnt, int64_t world, int64_t my_rank, torch::Tensor my_off, torch::Tensor m_block_expert,
                torch::Tensor num_blocks, int64_t align) {
  TORCH_CHECK(cnt.is_contiguous() && cnt.scalar_type() == at::kInt && cnt.size(0) == world);
  CKP(cb::moe_layout(cnt.data_ptr<int>(), world, cnt.size(1), my_rank, m_block_expert.numel(), int(align),
                     my_off.data_ptr<int>(), m_block_expert.data_ptr<int>(), num_blocks.data_ptr<int>(), stream()));
}
void moe_dispatch(torch::Tensor x, torch::Tensor ids, int64_t El, int64_t my_rank, torch::Tensor pair_rank,
                  torch::Tensor recv_ptrs, torch::Tensor sf_ptrs, torch::Tensor my_off,
                  c10::optional<torch::Tensor> rinfo_ptrs, int64_t cap, torch::Tensor pos_out, torch::Tensor status) {
  TORCH_CHECK(x.is_contiguous() && x.scalar_type() == at::kBFloat16);
  CKP(cb::moe_dispatch(x.data_ptr(), x.size(0), x.size(1), ids.data_ptr<int>(), ids.size(1), El, my_rank,
                       pair_rank.data_ptr<int>(), u64(recv_ptrs), u64(sf_ptrs), my_off.data_ptr<int>(),
                       rinfo_ptrs.has_value() && rinfo_ptrs->defined() ? u64(*rinfo_ptrs) : nullptr, cap,
                       pos_out.data_ptr<int>(), status.data_ptr<int>(), stream()));
}
void moe_combine_slots(torch::Tensor slots, torch::Tensor pos, torch::Tensor w, c10::optional<torch::Tensor> add,
                       torch::Tensor out) {
  TORCH_CHECK(slots.is_contiguous() && slots.scalar_type() == at::kBFloat16 && out.is_contiguous());
  TORCH_CHECK(pos.is_contiguous() && w.is_contiguous() && slots.size(0) >= pos.numel());
  CKP(cb::moe_combine_slots(slots.data_ptr(), out.size(0), out.size(1), pos.data_ptr<int>(), w.data_ptr<float>(),
                            pos.size(1), add.has_value() && add->defined() ? add->data_ptr() : nullptr,
                            out.data_ptr(), stream()));
}
// Grouped expert down-projection whose output rows are pushed to the tokens' home ranks (EP combine).
void gemm_fp8_push(torch::Tensor A, torch::Tensor sfa, torch::Tensor B, torch::Tensor sfb, torch::Tensor mbe,
                   torch::Tensor nb, int64_t n_per_group, torch::Tensor row_dst, torch::Tensor home_ptrs,
                   torch::Tensor status) {
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && A.scalar_type() == at::kFloat8_e4m3fn &&
              B.scalar_type() == at::kFloat8_e4m3fn && A.size(1) == B.size(1));
  TORCH_CHECK(row_dst.numel() >= A.size(0) && row_dst.scalar_type() == at::kInt);
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  CKP(cb::gemm_fp8_push(A.data_ptr(), B.data_ptr(), reinterpret_cast<const uint32_t*>(sfa.data_ptr()),
                        reinterpret_cast<const uint32_t*>(sfb.data_ptr()), A.size(0), n_per_group, A.size(1),
                        B.size(0), mbe.data_ptr<int>(), nb.data_ptr<int>(), mbe.numel(), row_dst.data_ptr<int>(),
                        u64(home_ptrs), home_ptrs.numel(), status.data_ptr<int>(), sms, stream()));
}
void moe_combine_pull(torch::Tensor y_ptrs, torch::Tensor ids, torch::Tensor pos, torch::Tensor w, int64_t El,
                      c10::optional<torch::Tensor> add, torch::Tensor out) {
  CKP(cb::moe_combine_pull(u64(y_ptrs), out.size(0), out.size(1), ids.data_ptr<int>(), pos.data_ptr<int>(),
                           w.data_ptr<float>(), ids.size(1), El,
                           add.has_value() && add->defined() ? add->data_ptr() : nullptr, out.data_ptr(), stream()));
}
void embed_peer(torch::Tensor table_ptrs, int64_t per, torch::Tensor ids, torch::Tensor X,
                c10::optional<torch::Tensor> sumsq) {
  CKP(cb::embed_peer(u64(table_ptrs), per, table_ptrs.numel(), ids.data_ptr<int>(), ids.numel(), X.size(2), X.size(1),
                     X.data_ptr(), sumsq.has_value() ? sumsq->data_ptr<float>() : nullptr, stream()));
}

// o_proj GEMM -> reduce-scatter: A fp8 [M,K] + SF tiles, W fp8 [N,K] + SF tiles; rows go to their owners' slots.
void gemm_fp8_scatter(torch::Tensor A, torch::Tensor sfa, torch::Tensor B, torch::Tensor sfb, torch::Tensor slot_ptrs,
                      torch::Tensor bounds, int64_t my_rank, int64_t slot_rows, torch::Tensor status) {
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && A.scalar_type() == at::kFloat8_e4m3fn &&
              B.scalar_type() == at::kFloat8_e4m3fn && A.size(1) == B.size(1));
  int dev;
  cudaGetDevice(&dev);
  int sms;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  CKP(cb::gemm_fp8_scatter(A.data_ptr(), B.data_ptr(), reinterpret_cast<const uint32_t*>(sfa.data_ptr()),
                           reinterpret_cast<const uint32_t*>(sfb.data_ptr()), A.size(0), B.size(0), A.size(1),
                           u64(slot_ptrs), bounds.data_ptr<int>(), slot_ptrs.numel(), my_rank, slot_rows,
                           status.data_ptr<int>(), sms, stream()));
}

}  // namespace

void register_p2p(pybind11::module_& m) {
  m.def("symm_malloc", &symm_malloc);
  m.def("symm_free", &symm_free);
  m.def("symm_ipc_handle", &symm_ipc_handle);
  m.def("symm_ipc_open", &symm_ipc_open);
  m.def("symm_ipc_close", &symm_ipc_close);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("signal_peers", &signal_peers);
  m.def("wait_flags", &wait_flags);
  m.def("p2p_barrier", &p2p_barrier);
  m.def("p2p_gather_rows", &p2p_gather_rows);
  m.def("p2p_scatter_partials", &p2p_scatter_partials);
  m.def("reduce_slots", &reduce_slots);
  m.def("p2p_a2a_heads", &p2p_a2a_heads);
  m.def("moe_count", &moe_count);
  m.def("moe_layout", &moe_layout);
  m.def("moe_combine_slots", &moe_combine_slots);
  m.def("gemm_fp8_push", &gemm_fp8_push);
  m.def("moe_dispatch", &moe_dispatch);
  m.def("moe_combine_pull", &moe_combine_pull);
  m.def("embed_peer", &embed_peer);
  m.def("gemm_fp8_scatter", &gemm_fp8_scatter);
}
