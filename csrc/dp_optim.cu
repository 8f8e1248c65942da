// Data-parallel distributed optimizer step fused with its collectives, over
// NVLink peer memory (every DP rank's fp32 gradient buffer and bf16 parameter
// buffer are mapped on every GPU of the node through CUDA IPC).
//
// dp_reduce_shard:   grad_shard[i] = sum_r grad_r[lo + i] (ranks summed in rank
//                    order, so every rank reduces its shard with identical bits),
//                    plus per-CTA partial sums of squares for the clip norm:
//                    the reduce-scatter, fused with the norm's first pass.
// dp_adam_allgather: AdamW on this rank's fp32 master shard (decoupled weight
//                    decay except on the listed no-decay ranges; bias corrections
//                    folded into host scalars; clip scale applied to the
//                    gradient) and the new bf16 weights stored into EVERY DP
//                    rank's parameter buffer at the shard's offset: the update
//                    fused with the parameter all-gather.
//
// Reference counterpart: MCore DistributedOptimizer (grad reduce-scatter, fp32
// Adam on the shard, parameter all-gather; nemo_rl config keys
// use_distributed_optimizer / overlap_grad_reduce / overlap_param_gather).
// Both kernels need the surrounding stream-ordered fences that the host code
// places: peers finished writing gradients before dp_reduce_shard, and every
// rank's dp_adam_allgather finished before anyone reads its parameters.
#include "common.cuh"

namespace rlb {
namespace dpo {

constexpr int kMaxRanks = 8;
struct Ptrs {
  const float* g[kMaxRanks];
  __nv_bfloat16* p[kMaxRanks];
};

__global__ void __launch_bounds__(256)
reduce_shard_kernel(Ptrs ptrs, int n, long long lo, long long len4, float* __restrict__ out,
                    float* __restrict__ part) {
  __shared__ float red[32];
  float sq = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < len4; i += (long long)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    // rank-ordered sum: loads from all peers are issued before the adds
    float4 v[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < n) v[r] = __ldcs(reinterpret_cast<const float4*>(ptrs.g[r] + lo) + i);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < n) {
        acc.x += v[r].x;
        acc.y += v[r].y;
        acc.z += v[r].z;
        acc.w += v[r].w;
      }
    reinterpret_cast<float4*>(out)[i] = acc;
    sq += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  sq = block_sum(sq, red);
  if (threadIdx.x == 0) part[blockIdx.x] = sq;
}

// no-decay ranges [R][2] (shard-local element offsets, sorted, disjoint,
// multiples of 4), staged in shared memory; binary search per 4-element vector
__global__ void __launch_bounds__(256)
adam_allgather_kernel(Ptrs ptrs, int n, long long lo, long long len4, float* __restrict__ master,
                      const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                      const long long* __restrict__ nodecay, int R, float lr, float b1, float b2, float eps, float wd,
                      float step_size, float inv_bc2_sqrt, float gscale) {
  extern __shared__ long long snd[];
  for (int i = threadIdx.x; i < 2 * R; i += blockDim.x) snd[i] = nodecay[i];
  __syncthreads();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < len4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = i * 4;
    int a = 0, b = R;  // first range whose end > e
    while (a < b) {
      const int mid = (a + b) >> 1;
      if (snd[2 * mid + 1] <= e) a = mid + 1;
      else b = mid;
    }
    const bool decayed = !(a < R && snd[2 * a] <= e);
    const float wdi = decayed ? wd : 0.f;
    float4 pp = reinterpret_cast<float4*>(master)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    const float4 gg4 = reinterpret_cast<const float4*>(g)[i];
    const float gg[4] = {gg4.x * gscale, gg4.y * gscale, gg4.z * gscale, gg4.w * gscale};
    float* P = &pp.x;
    float* M = &mm.x;
    float* V = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      M[k] = b1 * M[k] + (1.f - b1) * gg[k];
      V[k] = b2 * V[k] + (1.f - b2) * gg[k] * gg[k];
      const float denom = sqrtf(V[k]) * inv_bc2_sqrt + eps;
      P[k] = P[k] * (1.f - lr * wdi) - step_size * M[k] / denom;
    }
    reinterpret_cast<float4*>(master)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(P[0], P[1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(P[2], P[3]);
    uint2 packed;
    packed.x = *reinterpret_cast<uint32_t*>(&h0);
    packed.y = *reinterpret_cast<uint32_t*>(&h1);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < n) reinterpret_cast<uint2*>(ptrs.p[r] + lo)[i] = packed;
  }
}

// Readiness of gradient buckets for the reduction overlapped with the backward
// pass: every rank stores the step's epoch into its word `idx` of a symmetric
// u32 array (a stream memory write after the bucket's last gradient kernel);
// the reducing rank's side stream runs wait_ready_kernel (one thread per rank,
// acquire loads at system scope, bounded by the peer-wait budget; on expiry it
// sets the error word to 1000 + idx and returns) and then reduce_shard_kernel
// over the bucket's part of its shard.
__device__ int g_dpo_error = 0;

struct FlagPtrs {
  const uint32_t* f[kMaxRanks];
};

__global__ void wait_ready_kernel(FlagPtrs fp, int n, int idx, uint32_t epoch, long long limit) {
  const int r = threadIdx.x;
  if (r >= n) return;
  const uint32_t* p = fp.f[r] + idx;
  const long long t0 = clock64();
  for (;;) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    if ((int)(v - epoch) >= 0) return;
    if (clock64() - t0 > limit) {
      atomicExch(&g_dpo_error, 1000 + idx);
      return;
    }
    __nanosleep(200);
  }
}

}  // namespace dpo
}  // namespace rlb

using namespace rlb;

void dp_wait_ready(std::vector<int64_t> flag_ptrs, int64_t idx, int64_t epoch) {
  TORCH_CHECK(!flag_ptrs.empty() && flag_ptrs.size() <= (size_t)dpo::kMaxRanks, "dp_wait_ready: 1..8 ranks");
  dpo::FlagPtrs fp{};
  for (size_t i = 0; i < flag_ptrs.size(); ++i) fp.f[i] = reinterpret_cast<const uint32_t*>((uintptr_t)flag_ptrs[i]);
  // the budget covers the skew of one micro-batch's backward between the ranks
  dpo::wait_ready_kernel<<<1, 32, 0, stream()>>>(fp, (int)flag_ptrs.size(), (int)idx, (uint32_t)epoch,
                                                 4 * peer_wait_cycles());
  RLB_CUDA_CHECK(cudaGetLastError());
}

int64_t dp_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, dpo::g_dpo_error, sizeof(int)));
  if (reset && v) {
    const int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(dpo::g_dpo_error, &z, sizeof(int)));
  }
  return v;
}

namespace {
dpo::Ptrs make_ptrs(const std::vector<int64_t>& g, const std::vector<int64_t>& p) {
  TORCH_CHECK(!g.empty() && g.size() <= (size_t)dpo::kMaxRanks, "dp optimizer: 1..8 ranks");
  dpo::Ptrs s{};
  for (size_t i = 0; i < g.size(); ++i) {
    TORCH_CHECK(g[i] % 16 == 0, "dp optimizer: gradient buffers must be 16-byte aligned");
    s.g[i] = reinterpret_cast<const float*>((uintptr_t)g[i]);
  }
  for (size_t i = 0; i < p.size(); ++i) {
    TORCH_CHECK(p[i] % 16 == 0, "dp optimizer: parameter buffers must be 16-byte aligned");
    s.p[i] = reinterpret_cast<__nv_bfloat16*>((uintptr_t)p[i]);
  }
  return s;
}
int grid_for(long long len4) {
  return (int)std::max<long long>(1, std::min<long long>((len4 + 255) / 256, (long long)num_sms() * 8));
}
}  // namespace

// Returns the per-CTA partial sums of squares (fp32 [grid]); out: fp32 [len].
at::Tensor dp_reduce_shard(std::vector<int64_t> grad_ptrs, int64_t lo, int64_t len, at::Tensor out) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == len,
              "dp_reduce_shard: out must be fp32 [len]");
  TORCH_CHECK(lo % 4 == 0 && len % 4 == 0, "dp_reduce_shard: shard offset / length must be multiples of 4");
  const c10::cuda::CUDAGuard guard(out.device());
  const long long len4 = len / 4;
  const int grid = grid_for(len4);
  auto part = at::empty({grid}, out.options());
  dpo::reduce_shard_kernel<<<grid, 256, 0, stream()>>>(make_ptrs(grad_ptrs, {}), (int)grad_ptrs.size(), lo, len4,
                                                       out.data_ptr<float>(), part.data_ptr<float>());
  RLB_CUDA_CHECK(cudaGetLastError());
  return part;
}

void dp_adam_allgather(std::vector<int64_t> param_ptrs, int64_t lo, at::Tensor master, at::Tensor grad,
                       at::Tensor exp_avg, at::Tensor exp_avg_sq, at::Tensor nodecay, double lr, double b1, double b2,
                       double eps, double wd, int64_t step, double gscale) {
  const long long len = master.numel();
  TORCH_CHECK(master.is_cuda() && grad.numel() == len && exp_avg.numel() == len && exp_avg_sq.numel() == len,
              "dp_adam_allgather: shard tensors must match");
  TORCH_CHECK(lo % 4 == 0 && len % 4 == 0, "dp_adam_allgather: shard offset / length must be multiples of 4");
  TORCH_CHECK(nodecay.is_cuda() && nodecay.scalar_type() == at::kLong && nodecay.dim() == 2 && nodecay.size(1) == 2,
              "dp_adam_allgather: nodecay int64 [R, 2]");
  const int R = (int)nodecay.size(0);
  TORCH_CHECK(R <= 3072, "dp_adam_allgather: too many no-decay ranges (max 3072)");
  const c10::cuda::CUDAGuard guard(master.device());
  std::vector<int64_t> none(param_ptrs.size(), 16);
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  const long long len4 = len / 4;
  const int smem = std::max(16, 2 * R * 8);
  dpo::adam_allgather_kernel<<<grid_for(len4), 256, smem, stream()>>>(
      make_ptrs(none, param_ptrs), (int)param_ptrs.size(), lo, len4, master.data_ptr<float>(),
      grad.data_ptr<float>(), exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(),
      reinterpret_cast<const long long*>(nodecay.data_ptr<int64_t>()), R,
      (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)(lr / bc1), (float)(1.0 / std::sqrt(bc2)),
      (float)gscale);
  RLB_CUDA_CHECK(cudaGetLastError());
}
