// MoE router: softmax over the experts, top-k selection and the expert-grouped
// permutation of the token -> expert assignments, in three small kernels.
//
//   router_topk_kernel   one warp per token: the fp32 logits row in registers,
//                        warp max / sum for the softmax (probabilities written),
//                        k rounds of a warp arg-max (ties -> the lower expert id),
//                        and a per-block histogram of the chosen experts.
//   router_scan_kernel   one CTA per expert: an exclusive scan of the block
//                        histograms over the blocks (each block's first slot
//                        inside the expert's range) and the expert total.
//   router_pos_kernel    per block, the experts' first rows (a scan of the totals
//                        in shared memory), then each assignment's rank among the
//                        block's earlier assignments to the same expert; its row in
//                        the expert-grouped order is expert start + block start + rank.
//
// The result is the stable sort of the flattened [T*k] expert ids (the order a
// stable argsort gives): assignments grouped by expert, in token order inside an
// expert, so the grouped expert GEMM sees a deterministic row order.
//
// Reference counterpart: the router top-k and token permutation of Transformer
// Engine's MoE path that MCore calls; the reference patches TE's Triton
// permutation kernel (nemo_rl/models/policy/workers/patches.py:56).
#include "common.cuh"

namespace rlb {
namespace router {

constexpr int kWarps = 16;  // tokens per block of the top-k and position kernels

template <int NPL>
__global__ void __launch_bounds__(kWarps * 32)
router_topk_kernel(const float* __restrict__ logits, int T, int E, int k, float* __restrict__ probs,
                   int64_t* __restrict__ ids, int* __restrict__ block_counts) {
  extern __shared__ int s_cnt[];  // [E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  const long long t = (long long)blockIdx.x * kWarps + warp;
  if (t < T) {
    const float* row = logits + t * E;
    float v[NPL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? row[e] : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? expf(v[i] - mx) : 0.f;
      s += v[i];
    }
    s = warp_sum(s);
    const float inv = 1.f / s;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? v[i] * inv : -1.f;  // padding lanes never win
      if (e < E) probs[t * E + e] = v[i];
    }
    for (int j = 0; j < k; ++j) {
      float best = -2.f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int e = lane + 32 * i;
        if (v[i] > best || (v[i] == best && e < bi)) {
          best = v[i];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      if (lane == 0) {
        ids[t * k + j] = bi;
        atomicAdd(&s_cnt[bi], 1);
      }
#pragma unroll
      for (int i = 0; i < NPL; ++i)
        if (bi == lane + 32 * i) v[i] = -1.f;  // taken (probabilities are >= 0)
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_counts[(long long)blockIdx.x * E + e] = s_cnt[e];
}

// One block per expert: exclusive scan of the expert's per-block counts over the
// blocks (each thread sums a contiguous run of blocks, a shared-memory scan of
// the run totals, then each thread writes its run's bases) and the expert total.
constexpr int kScanThreads = 256;

__global__ void __launch_bounds__(kScanThreads)
router_scan_kernel(int* __restrict__ block_counts, int nblk, int E, int* __restrict__ counts) {
  __shared__ int s_run[kScanThreads];
  const int e = blockIdx.x, t = threadIdx.x;
  const int per = (nblk + kScanThreads - 1) / kScanThreads;
  const int b0 = t * per, b1 = min(nblk, b0 + per);
  int sum = 0;
  for (int b = b0; b < b1; ++b) sum += block_counts[(long long)b * E + e];
  s_run[t] = sum;
  __syncthreads();
  // inclusive Hillis-Steele scan of the run totals
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const int v = t >= off ? s_run[t - off] : 0;
    __syncthreads();
    s_run[t] += v;
    __syncthreads();
  }
  int run = t == 0 ? 0 : s_run[t - 1];
  for (int b = b0; b < b1; ++b) {
    int* p = block_counts + (long long)b * E + e;
    const int c = *p;
    *p = run;
    run += c;
  }
  if (t == kScanThreads - 1) counts[e] = s_run[t];
}

__global__ void __launch_bounds__(256)
router_pos_kernel(const int64_t* __restrict__ ids, long long TK, int k, int E, const int* __restrict__ block_base,
                  const int* __restrict__ counts, int64_t* __restrict__ order, int64_t* __restrict__ pos) {
  extern __shared__ int s_mem[];  // [E] expert starts, then the block's assignments' experts
  int* expert_start = s_mem;
  int* s_e = s_mem + E;
  const long long a0 = (long long)blockIdx.x * kWarps * k;
  const int n = (int)min((long long)kWarps * k, TK - a0);
  for (int i = threadIdx.x; i < n; i += blockDim.x) s_e[i] = (int)ids[a0 + i];
  for (int x = threadIdx.x; x < E; x += blockDim.x) expert_start[x] = counts[x];
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive scan of the expert totals in shared memory (E <= 1024)
    int acc = 0;
    for (int x = 0; x < E; ++x) {
      const int c = expert_start[x];
      expert_start[x] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = s_e[i];
    int r = 0;
    for (int j = 0; j < i; ++j) r += (s_e[j] == e);
    const long long p = (long long)expert_start[e] + block_base[(long long)blockIdx.x * E + e] + r;
    if (!RLB_IN_BOUNDS(p, TK, kBoundsRouterRow)) continue;
    order[p] = a0 + i;
    pos[a0 + i] = p;
  }
}

template <int NPL>
void launch_topk(const float* logits, int T, int E, int k, float* probs, int64_t* ids, int* bc, int nblk) {
  router_topk_kernel<NPL><<<nblk, kWarps * 32, E * sizeof(int), stream()>>>(logits, T, E, k, probs, ids, bc);
}

}  // namespace router
}  // namespace rlb

// logits [T, E] fp32 -> (probs [T, E] fp32, ids [T, k] int64, counts [E] int32,
// order [T*k] int64: assignment index at each expert-grouped row, pos [T*k] int64:
// the inverse (row of each assignment)).
std::vector<at::Tensor> moe_router_topk(at::Tensor logits, int64_t k) {
  using namespace rlb;
  using namespace rlb::router;
  RLB_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.scalar_type() == at::kFloat && logits.is_contiguous(),
            "moe_router_topk: logits must be a contiguous fp32 [T, E] CUDA tensor");
  const int T = logits.size(0), E = logits.size(1);
  RLB_CHECK(E >= 1 && E <= 1024, "moe_router_topk: 1 <= experts <= 1024");
  RLB_CHECK(k >= 1 && k <= E && k <= 64, "moe_router_topk: 1 <= k <= min(experts, 64)");
  const c10::cuda::CUDAGuard g(logits.device());
  auto o32 = logits.options().dtype(at::kInt), o64 = logits.options().dtype(at::kLong);
  auto probs = at::empty({T, E}, logits.options());
  auto ids = at::empty({T, k}, o64);
  auto counts = at::zeros({E}, o32);
  auto order = at::empty({(long long)T * k}, o64);
  auto pos = at::empty({(long long)T * k}, o64);
  if (T == 0) return {probs, ids, counts, order, pos};
  const int nblk = (T + kWarps - 1) / kWarps;
  auto bc = at::empty({nblk, E}, o32);
  const float* lp = logits.data_ptr<float>();
  float* pp = probs.data_ptr<float>();
  int64_t* ip = ids.data_ptr<int64_t>();
  int* bp = bc.data_ptr<int>();
  const int npl = (E + 31) / 32;
  if (npl <= 1) launch_topk<1>(lp, T, E, k, pp, ip, bp, nblk);
  else if (npl <= 2) launch_topk<2>(lp, T, E, k, pp, ip, bp, nblk);
  else if (npl <= 4) launch_topk<4>(lp, T, E, k, pp, ip, bp, nblk);
  else if (npl <= 8) launch_topk<8>(lp, T, E, k, pp, ip, bp, nblk);
  else if (npl <= 16) launch_topk<16>(lp, T, E, k, pp, ip, bp, nblk);
  else launch_topk<32>(lp, T, E, k, pp, ip, bp, nblk);
  RLB_CUDA_CHECK(cudaGetLastError());
  router_scan_kernel<<<E, kScanThreads, 0, stream()>>>(bp, nblk, E, counts.data_ptr<int>());
  RLB_CUDA_CHECK(cudaGetLastError());
  router_pos_kernel<<<nblk, 256, (E + kWarps * k) * sizeof(int), stream()>>>(
      ip, (long long)T * k, (int)k, E, bp, counts.data_ptr<int>(), order.data_ptr<int64_t>(), pos.data_ptr<int64_t>());
  RLB_CUDA_CHECK(cudaGetLastError());
  return {probs, ids, counts, order, pos};
}

int64_t bounds_error_moe_router(bool reset) { return rlb::rlb_bounds_error(reset); }
