// NVLink SHARP (NVLS) collectives through NVSwitch multicast memory.
//
// A multicast object binds one equal-sized allocation of every rank of a group;
// a load from the multicast address with multimem.ld_reduce returns the SUM of
// all ranks' values at that offset (the reduction runs in the switch), and a
// multimem.st writes one value to every rank's allocation.  So:
//
//   nvls_all_reduce:     rank r reduces slice r of the buffer (ld_reduce) and
//                        stores the sums back through the multicast address, so
//                        every rank ends with the full sum; each element crosses
//                        NVLink once towards the switch per rank and once back.
//   nvls_reduce_shard:   rank r reduces [lo, lo + len) and writes the sums to a
//                        local output (a reduce-scatter when each rank asks for
//                        its own shard).
//   nvls_barrier:        one thread per peer: release-store the call's epoch into
//                        that peer's signal word for this rank, then acquire-poll
//                        this rank's word of every peer until it reaches the epoch
//                        (bounded by the peer-wait budget; on expiry the error word
//                        is set and the kernel returns).
//
// Ordering: a barrier before the reduction (every rank's inputs are written and
// fenced) and one after it (no rank reads or rewrites its buffer while a peer's
// multicast stores may still be landing).  Loads / stores are .relaxed at system
// scope; the barriers carry the ordering (fence + release / acquire).
//
// Reference counterpart: NCCL's NVLS all-reduce / reduce-scatter that MCore's
// collectives use on NVSwitch systems.
#include "common.cuh"

namespace rlb {
namespace nvls {

__device__ int g_nvls_error = 0;
constexpr int kMaxRanks = 8;

struct Pads {
  uint32_t* pad[kMaxRanks];  // every rank's signal words (this rank's slot for peer p at index p)
};

__global__ void barrier_kernel(Pads pads, int world, int rank, uint32_t epoch, long long limit) {
  const int p = threadIdx.x;
  if (p >= world) return;
  __threadfence_system();  // this rank's earlier writes are visible before the signal
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(pads.pad[p] + rank), "r"(epoch) : "memory");
  const uint32_t* mine = pads.pad[rank] + p;
  const long long t0 = clock64();
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(mine) : "memory");
    if ((int)(v - epoch) >= 0) break;
    if (clock64() - t0 > limit) {
      atomicExch(&g_nvls_error, 1 + p);
      return;
    }
    __nanosleep(100);
  }
}

__device__ __forceinline__ uint4 ld_reduce_bf16(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_reduce_f32(const void* mc) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_mc_bf16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};\n" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void st_mc_f32(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// 16-byte vectors [v0, v1) of the multicast buffer: reduced; stored back through
// the multicast address (out == nullptr) or into out[v - v0].  Each thread keeps
// kUnroll independent reductions in flight (the switch round trip is long).
constexpr int kUnroll = 4;

template <bool F32>
__global__ void __launch_bounds__(512) reduce_kernel(char* mc, long long v0, long long v1, uint4* out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long base = v0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; base < v1;
       base += stride * kUnroll) {
    uint4 s[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long v = base + u * stride;
      if (v < v1) s[u] = F32 ? ld_reduce_f32(mc + v * 16) : ld_reduce_bf16(mc + v * 16);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long v = base + u * stride;
      if (v >= v1) break;
      if (out == nullptr) {
        if (F32) st_mc_f32(mc + v * 16, s[u]);
        else st_mc_bf16(mc + v * 16, s[u]);
      } else {
        out[v - v0] = s[u];
      }
    }
  }
}

Pads make_pads(const std::vector<int64_t>& pads) {
  TORCH_CHECK(!pads.empty() && pads.size() <= (size_t)kMaxRanks, "nvls: 1..8 ranks");
  Pads p{};
  for (size_t i = 0; i < pads.size(); ++i) p.pad[i] = reinterpret_cast<uint32_t*>((uintptr_t)pads[i]);
  return p;
}

void launch_reduce(int64_t mc_ptr, long long v0, long long v1, bool f32, uint4* out) {
  if (v1 <= v0) return;
  const long long per_cta = 512LL * kUnroll;
  const int grid = (int)std::max<long long>(1, std::min<long long>((v1 - v0 + per_cta - 1) / per_cta,
                                                                    (long long)num_sms() * 4));
  char* mc = reinterpret_cast<char*>((uintptr_t)mc_ptr);
  if (f32) reduce_kernel<true><<<grid, 512, 0, stream()>>>(mc, v0, v1, out);
  else reduce_kernel<false><<<grid, 512, 0, stream()>>>(mc, v0, v1, out);
  RLB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace nvls
}  // namespace rlb

using namespace rlb;

void nvls_barrier(std::vector<int64_t> pad_ptrs, int64_t rank, int64_t epoch) {
  const int world = (int)pad_ptrs.size();
  TORCH_CHECK(rank >= 0 && rank < world, "nvls_barrier: bad rank");
  nvls::barrier_kernel<<<1, 32, 0, stream()>>>(nvls::make_pads(pad_ptrs), world, (int)rank, (uint32_t)epoch,
                                               peer_wait_cycles());
  RLB_CUDA_CHECK(cudaGetLastError());
}

// In-place sum over the group of `nbytes` bytes (fp32 or bf16) at the multicast
// address; every rank reduces its 1/world slice.  nbytes must be a multiple of
// 16 * world; the caller brackets the call with nvls_barrier.
void nvls_all_reduce(int64_t mc_ptr, int64_t nbytes, bool f32, int64_t rank, int64_t world) {
  TORCH_CHECK(mc_ptr % 16 == 0 && nbytes % (16 * world) == 0, "nvls_all_reduce: 16-byte vectors per rank slice");
  const long long nv = nbytes / 16, per = nv / world;
  nvls::launch_reduce(mc_ptr, rank * per, (rank + 1) * per, f32, nullptr);
}

// Sum over the group of bytes [lo, lo + len) at the multicast address into `out`
// (local, contiguous, `len` bytes).
void nvls_reduce_shard(int64_t mc_ptr, int64_t lo, int64_t len, at::Tensor out, bool f32) {
  TORCH_CHECK(out.is_cuda() && out.is_contiguous() && out.nbytes() == (size_t)len, "nvls_reduce_shard: out size");
  TORCH_CHECK((mc_ptr + lo) % 16 == 0 && len % 16 == 0 && out.data_ptr() != nullptr &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "nvls_reduce_shard: 16-byte aligned offsets and length");
  const c10::cuda::CUDAGuard g(out.device());
  nvls::launch_reduce(mc_ptr + lo, 0, len / 16, f32, reinterpret_cast<uint4*>(out.data_ptr()));
}

int64_t nvls_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, nvls::g_nvls_error, sizeof(int)));
  if (reset && v) {
    const int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(nvls::g_nvls_error, &z, sizeof(int)));
  }
  return v;
}
