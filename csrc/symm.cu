// Symmetric device memory across the ranks of one node (CUDA IPC).
//
// Every rank allocates the same-sized buffer with cudaMalloc, exports its IPC
// handle, and (after the handles are exchanged over the process group) opens
// every peer's handle, so kernels can load and store peer HBM directly over
// NVLink / NVSwitch.  The library keeps the raw allocations (outside torch's
// caching allocator, whose blocks cannot be exported individually).
#include "common.cuh"

#include <mutex>
#include <unordered_map>

namespace {
std::mutex g_mu;
std::unordered_map<uint64_t, void*> g_local;   // ptr -> base (own allocations)
std::unordered_map<uint64_t, void*> g_opened;  // ptr -> opened peer mapping
}  // namespace

// Allocate `bytes` of zeroed device memory; returns (ptr, ipc handle bytes).
std::tuple<int64_t, at::Tensor> symm_alloc(int64_t bytes) {
  TORCH_CHECK(bytes > 0, "symm_alloc: bytes must be positive");
  void* p = nullptr;
  RLB_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  RLB_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  RLB_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto t = at::empty({(int64_t)sizeof(h)}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  std::lock_guard<std::mutex> lk(g_mu);
  g_local[(uint64_t)p] = p;
  return {(int64_t)(uintptr_t)p, t};
}

// Open a peer's exported handle; returns the mapped device pointer.
int64_t symm_open(at::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "symm_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  RLB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  std::lock_guard<std::mutex> lk(g_mu);
  g_opened[(uint64_t)p] = p;
  return (int64_t)(uintptr_t)p;
}

void symm_close(int64_t ptr) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_opened.find((uint64_t)ptr);
  if (it != g_opened.end()) {
    cudaIpcCloseMemHandle(it->second);
    g_opened.erase(it);
    return;
  }
  auto jt = g_local.find((uint64_t)ptr);
  if (jt != g_local.end()) {
    cudaFree(jt->second);
    g_local.erase(jt);
  }
}

// View `numel` elements of `dtype` at device address `ptr` as a tensor (no copy,
// no ownership): the caller keeps the symmetric buffer alive.
at::Tensor symm_view(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device) {
  auto dt = static_cast<at::ScalarType>(dtype_code);
  auto opts = at::TensorOptions().dtype(dt).device(at::kCUDA, device);
  return at::from_blob(reinterpret_cast<void*>((uintptr_t)ptr), {numel}, [](void*) {}, opts);
}
