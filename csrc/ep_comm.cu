// Expert-parallel token exchange over NVLink peer memory (MoE dispatch / combine).
//
// ep_scatter: every item i moves one bf16 row of H elements (row src_row[i] of
//   this rank's source matrix, or row i when src_row is null) straight into
//   row dst_row[i] of rank dst_rank[i]'s receive buffer (peer stores), and
//   optionally stores a 32-bit tag beside it (the receiver learns where each
//   row came from).  Dispatch uses it with the rows already placed at their
//   final, expert-grouped positions, so the receiver needs no permutation;
//   combine uses it to return expert outputs to the slot of the assignment that
//   produced them.
// ep_consume: waits until every source rank has finished its scatter of this
//   epoch, copies the first `rows` received rows (and tags) out of the receive
//   buffer and acknowledges the epoch to every source, which may then reuse the
//   slot (receive buffers are double-buffered by epoch parity).
//
// Flow control, all in the symmetric flag words of each rank ([2][n] u32 each):
//   data flags   flags_d[par][s] = epoch  written by source s after its stores to d
//   acks         acks_s[par][d]  = epoch  written by d after it consumed s's rows
// A scatter of epoch e first waits acks_me[par][d] >= e - 2 for every destination.
// Every wait is bounded (clock64 budget): on expiry an error word is set and the
// kernel returns (the host reads it with ep_error_flag).
//
// Reference counterpart: MCore's alltoall token dispatcher / DeepEP / HybridEP
// (examples/configs/recipes/llm/performance/grpo-qwen3-30ba3b-4n8g.yaml:25-29).
#include "common.cuh"

namespace rlb {
namespace ep {

__device__ int g_ep_error = 0;
constexpr int kMax = 8;

struct Peers {
  __nv_bfloat16* buf[kMax];  // receive buffer base of every rank ([2][cap][H] bf16)
  int* tag[kMax];            // tag base of every rank ([2][cap] int32)
  uint32_t* flags[kMax];     // data flags of every rank ([2][n])
  uint32_t* acks[kMax];      // ack words of every rank ([2][n])
  long long wait;            // bound of every wait on a peer's word (cycles)
};

__device__ __forceinline__ void st_rel(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acq(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ bool wait_ge(const uint32_t* p, uint32_t v, int code, long long limit) {
  const long long t0 = clock64();
  while ((int)(ld_acq(p) - v) < 0) {
    if (clock64() - t0 > limit) {
      atomicExch(&g_ep_error, code);
      return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(256)
scatter_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ src_row,
               const int* __restrict__ dst_rank, const int* __restrict__ dst_row, const int* __restrict__ tags,
               int n_items, int H, long long cap, Peers pe, int n, int me, uint32_t epoch,
               unsigned int* __restrict__ counter, long long src_rows) {
  __shared__ int ok;
  const int par = epoch & 1;
  if (threadIdx.x == 0) {
    bool good = true;
    if (epoch > 2)
      for (int d = 0; d < n && good; ++d) good = wait_ge(pe.acks[me] + par * n + d, epoch - 2, 1, pe.wait);
    ok = good;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int vpr = H / 8;  // 16-byte vectors per row
  if (ok) {
    for (int i = blockIdx.x * 8 + warp; i < n_items; i += gridDim.x * 8) {
      const int r = src_row ? src_row[i] : i;
      const int d = dst_rank[i];
      if (!RLB_IN_BOUNDS(r, src_rows, kBoundsEpRow) || !RLB_IN_BOUNDS(d, n, kBoundsEpRow) ||
          !RLB_IN_BOUNDS(dst_row[i], cap, kBoundsEpRow))
        continue;
      const long long row = (long long)par * cap + dst_row[i];
      const uint4* s = reinterpret_cast<const uint4*>(src + (long long)r * H);
      uint4* o = reinterpret_cast<uint4*>(pe.buf[d] + row * H);
      for (int c = lane; c < vpr; c += 32) o[c] = s[c];
      if (tags && lane == 0) pe.tag[d][row] = tags[i];
    }
  }
  // last CTA out publishes the epoch to every destination
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(counter + par, 1u);
    if (prev == gridDim.x - 1) {
      counter[par] = 0u;
      __threadfence_system();
      for (int d = 0; d < n; ++d) st_rel(pe.flags[d] + par * n + me, epoch);
    }
  }
}

__global__ void __launch_bounds__(256)
consume_kernel(Peers pe, int n, int me, uint32_t epoch, long long cap, int rows, int H,
               __nv_bfloat16* __restrict__ out, int* __restrict__ out_tag, unsigned int* __restrict__ counter) {
  __shared__ int ok;
  const int par = epoch & 1;
  if (threadIdx.x == 0) {
    bool good = true;
    for (int s = 0; s < n && good; ++s) good = wait_ge(pe.flags[me] + par * n + s, epoch, 2, pe.wait);
    ok = good;
  }
  __syncthreads();
  if (ok) {
    const long long nv = (long long)rows * (H / 8);
    const uint4* b = reinterpret_cast<const uint4*>(pe.buf[me] + (long long)par * cap * H);
    uint4* o = reinterpret_cast<uint4*>(out);
    for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < nv; v += (long long)gridDim.x * blockDim.x)
      o[v] = b[v];
    if (out_tag)
      for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < rows; j += (long long)gridDim.x * blockDim.x)
        out_tag[j] = pe.tag[me][(long long)par * cap + j];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(counter + 2 + par, 1u);
    if (prev == gridDim.x - 1) {
      counter[2 + par] = 0u;
      __threadfence_system();
      for (int s = 0; s < n; ++s) st_rel(pe.acks[s] + par * n + me, epoch);
    }
  }
}

}  // namespace ep
}  // namespace rlb

using namespace rlb;

namespace {
ep::Peers make_peers(const std::vector<int64_t>& buf, const std::vector<int64_t>& tag, const std::vector<int64_t>& flags,
                     const std::vector<int64_t>& acks) {
  const size_t n = buf.size();
  TORCH_CHECK(n >= 1 && n <= (size_t)ep::kMax && tag.size() == n && flags.size() == n && acks.size() == n,
              "ep: 1..8 ranks, one pointer per rank for every buffer");
  ep::Peers p{};
  p.wait = peer_wait_cycles();
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(buf[i] % 16 == 0, "ep: receive buffers must be 16-byte aligned");
    p.buf[i] = reinterpret_cast<__nv_bfloat16*>((uintptr_t)buf[i]);
    p.tag[i] = reinterpret_cast<int*>((uintptr_t)tag[i]);
    p.flags[i] = reinterpret_cast<uint32_t*>((uintptr_t)flags[i]);
    p.acks[i] = reinterpret_cast<uint32_t*>((uintptr_t)acks[i]);
  }
  return p;
}
}  // namespace

// src [R, H] bf16; src_row / dst_rank / dst_row / tags: int32 [n_items] (src_row,
// tags optional); counter: int32 [4] local, zero-initialised once.
void ep_scatter(at::Tensor src, c10::optional<at::Tensor> src_row, at::Tensor dst_rank, at::Tensor dst_row,
                c10::optional<at::Tensor> tags, int64_t cap, std::vector<int64_t> buf, std::vector<int64_t> tag,
                std::vector<int64_t> flags, std::vector<int64_t> acks, int64_t me, int64_t epoch, at::Tensor counter) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.dim() == 2,
              "ep_scatter: src bf16 [R, H]");
  const int H = src.size(1);
  TORCH_CHECK(H % 8 == 0, "ep_scatter: H % 8 == 0");
  TORCH_CHECK(dst_rank.scalar_type() == at::kInt && dst_row.scalar_type() == at::kInt, "ep_scatter: int32 maps");
  TORCH_CHECK(epoch >= 1, "ep_scatter: epochs start at 1");
  const int n_items = dst_rank.numel();
  const c10::cuda::CUDAGuard guard(src.device());
  const int grid = std::max(1, std::min((n_items + 7) / 8, num_sms() * 4));
  ep::scatter_kernel<<<grid, 256, 0, stream()>>>(
      (const __nv_bfloat16*)src.data_ptr(), src_row ? src_row->data_ptr<int>() : nullptr, dst_rank.data_ptr<int>(),
      dst_row.data_ptr<int>(), tags ? tags->data_ptr<int>() : nullptr, n_items, H, cap,
      make_peers(buf, tag, flags, acks), (int)buf.size(), (int)me, (uint32_t)epoch,
      reinterpret_cast<unsigned int*>(counter.data_ptr<int>()), (long long)src.size(0));
  RLB_CUDA_CHECK(cudaGetLastError());
}

void ep_consume(at::Tensor out, c10::optional<at::Tensor> out_tag, int64_t cap, std::vector<int64_t> buf,
                std::vector<int64_t> tag, std::vector<int64_t> flags, std::vector<int64_t> acks, int64_t me,
                int64_t epoch, at::Tensor counter) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.dim() == 2,
              "ep_consume: out bf16 [rows, H]");
  const int rows = out.size(0), H = out.size(1);
  TORCH_CHECK(rows <= cap && H % 8 == 0, "ep_consume: rows <= capacity, H % 8 == 0");
  const c10::cuda::CUDAGuard guard(out.device());
  const long long nv = (long long)rows * (H / 8);
  const int grid = (int)std::max<long long>(1, std::min<long long>((nv + 255) / 256, (long long)num_sms() * 4));
  ep::consume_kernel<<<grid, 256, 0, stream()>>>(make_peers(buf, tag, flags, acks), (int)buf.size(), (int)me,
                                                 (uint32_t)epoch, cap, rows, H, (__nv_bfloat16*)out.data_ptr(),
                                                 out_tag ? out_tag->data_ptr<int>() : nullptr,
                                                 reinterpret_cast<unsigned int*>(counter.data_ptr<int>()));
  RLB_CUDA_CHECK(cudaGetLastError());
}

int64_t ep_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, ep::g_ep_error, sizeof(int)));
  if (reset) {
    const int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(ep::g_ep_error, &z, sizeof(int)));
  }
  return v;
}

int64_t bounds_error_ep_comm(bool reset) { return rlb::rlb_bounds_error(reset); }
