// Speculative-decoding verification (rejection sampling) over the full vocabulary.
//
// For every sequence b with k draft tokens x_1..x_k, target logits t_i (rows
// i = 0..k: t_i scores the token after prefix + x_1..x_i) and draft logits d_i
// (i = 0..k-1, the distribution x_{i+1} was drawn from), both divided by the
// temperature:
//   for i = 0..k-1: accept x_{i+1} with probability min(1, p_i(x) / q_i(x));
//                   on rejection emit a token drawn from norm(max(0, p_i - q_i))
//                   and stop;
//   if all k are accepted, emit a bonus token drawn from p_k.
// The emitted sequence is distributed exactly as sampling token by token from
// the target (Leviathan et al. 2023; Chen et al. 2023).  Greedy mode
// (temperature 0) accepts while argmax p_i == x_{i+1} and emits argmax p_i.
//
// One CTA per sequence: block reductions over V for the max / sum-exp of each
// row, the acceptance test with a counter-based uniform, and Gumbel-max
// sampling (log residual + Gumbel noise) for the correction / bonus token.
// Outputs: tokens [B, k+1] (emitted tokens, -1 past the end), n_emit [B]
// (accepted + 1), and logprob [B, k+1] of each emitted token under p.
#include "common.cuh"

namespace rlb {
namespace spec {

constexpr int kThreads = 512;

struct MaxSum {
  float m, s;
};

__device__ __forceinline__ MaxSum merge(MaxSum a, MaxSum b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

template <typename T>
__device__ MaxSum row_lse(const T* __restrict__ row, int V, float inv_t, MaxSum* red) {
  MaxSum acc{-INFINITY, 0.f};
  for (int v = threadIdx.x; v < V; v += blockDim.x) acc = merge(acc, MaxSum{to_f(row[v]) * inv_t, 1.f});
  for (int o = 16; o > 0; o >>= 1) {
    MaxSum other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = merge(acc, other);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = acc;
  __syncthreads();
  if (w == 0) {
    acc = lane < (int)(blockDim.x >> 5) ? red[lane] : MaxSum{-INFINITY, 0.f};
    for (int o = 16; o > 0; o >>= 1) {
      MaxSum other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
      acc = merge(acc, other);
    }
    if (lane == 0) red[0] = acc;
  }
  __syncthreads();
  return red[0];
}

struct ArgMax {
  float v;
  int i;
};

__device__ __forceinline__ ArgMax amax(ArgMax a, ArgMax b) { return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a; }

__device__ ArgMax block_argmax(ArgMax x, ArgMax* red) {
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax other{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
    x = amax(x, other);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = x;
  __syncthreads();
  if (w == 0) {
    x = lane < (int)(blockDim.x >> 5) ? red[lane] : ArgMax{-INFINITY, 0x7fffffff};
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax other{__shfl_xor_sync(0xffffffffu, x.v, o), __shfl_xor_sync(0xffffffffu, x.i, o)};
      x = amax(x, other);
    }
    if (lane == 0) red[0] = x;
  }
  __syncthreads();
  return red[0];
}

// Gumbel(0,1) noise from the counter-based uniform
__device__ __forceinline__ float gumbel(uint32_t seed, uint32_t stream, uint32_t ctr) {
  return -__logf(-__logf(uniform01(seed, stream, ctr)));
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
verify_kernel(const T* __restrict__ tlog, const T* __restrict__ dlog, const long long* __restrict__ draft, int k,
              int V, float temperature, uint32_t seed, uint32_t offset, long long* __restrict__ out_tok,
              int* __restrict__ n_emit, float* __restrict__ out_lp) {
  __shared__ MaxSum red_ms[32];
  __shared__ ArgMax red_am[32];
  const int b = blockIdx.x;
  const bool greedy = temperature <= 0.f;
  const float inv_t = greedy ? 1.f : 1.f / temperature;
  const uint32_t stream_id = (uint32_t)b * 0x10001u + offset;
  int emitted = 0;
  bool stop = false;
  for (int i = 0; i <= k && !stop; ++i) {
    const T* tr = tlog + ((long long)b * (k + 1) + i) * V;
    const MaxSum tp = row_lse(tr, V, inv_t, red_ms);
    const float t_lse = tp.m + __logf(tp.s);
    int tok;
    if (i < k) {
      const int x = (int)draft[(long long)b * k + i];
      const T* dr = dlog + ((long long)b * k + i) * V;
      if (greedy) {
        ArgMax best{-INFINITY, 0x7fffffff};
        for (int v = threadIdx.x; v < V; v += blockDim.x) best = amax(best, ArgMax{to_f(tr[v]), v});
        best = block_argmax(best, red_am);
        tok = best.i;
        stop = tok != x;
      } else {
        const MaxSum dp = row_lse(dr, V, inv_t, red_ms);
        const float d_lse = dp.m + __logf(dp.s);
        const float lp_t = to_f(tr[x]) * inv_t - t_lse;
        const float lq = to_f(dr[x]) * inv_t - d_lse;
        const float u = uniform01(seed, stream_id, (uint32_t)(2 * i));
        if (__logf(u) < lp_t - lq) {
          tok = x;
        } else {
          // residual max(0, p - q): Gumbel-max over its logarithm
          ArgMax best{-INFINITY, 0x7fffffff};
          for (int v = threadIdx.x; v < V; v += blockDim.x) {
            const float p = __expf(to_f(tr[v]) * inv_t - t_lse);
            const float q = __expf(to_f(dr[v]) * inv_t - d_lse);
            const float r = p - q;
            if (r > 0.f) best = amax(best, ArgMax{__logf(r) + gumbel(seed, stream_id, (uint32_t)((2 * i + 1) * V + v)), v});
          }
          best = block_argmax(best, red_am);
          tok = best.i == 0x7fffffff ? x : best.i;  // p == q everywhere: nothing to correct
          stop = true;
        }
      }
    } else {
      // bonus token from p_k
      ArgMax best{-INFINITY, 0x7fffffff};
      for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float s = to_f(tr[v]) * inv_t;
        best = amax(best, ArgMax{greedy ? s : s + gumbel(seed, stream_id, (uint32_t)((2 * k + 1) * V + v)), v});
      }
      best = block_argmax(best, red_am);
      tok = best.i;
    }
    if (threadIdx.x == 0) {
      out_tok[(long long)b * (k + 1) + i] = tok;
      out_lp[(long long)b * (k + 1) + i] = to_f(tr[tok]) * inv_t - t_lse;
    }
    ++emitted;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    n_emit[b] = emitted;
    for (int i = emitted; i <= k; ++i) {
      out_tok[(long long)b * (k + 1) + i] = -1;
      out_lp[(long long)b * (k + 1) + i] = 0.f;
    }
  }
}

}  // namespace spec
}  // namespace rlb

using namespace rlb;

// target_logits [B, k+1, V], draft_logits [B, k, V] (same dtype), draft_tokens
// int64 [B, k]; returns (tokens int64 [B, k+1], n_emit int32 [B], logprobs fp32 [B, k+1]).
std::vector<at::Tensor> spec_verify(at::Tensor target_logits, at::Tensor draft_logits, at::Tensor draft_tokens,
                                    double temperature, int64_t seed, int64_t offset) {
  TORCH_CHECK(target_logits.is_cuda() && target_logits.dim() == 3 && target_logits.is_contiguous(),
              "spec_verify: target_logits [B, k+1, V] contiguous");
  const int B = target_logits.size(0), k = target_logits.size(1) - 1, V = target_logits.size(2);
  TORCH_CHECK(k >= 1, "spec_verify: at least one draft token");
  TORCH_CHECK(draft_logits.sizes() == at::IntArrayRef({B, k, V}) && draft_logits.is_contiguous() &&
                  draft_logits.scalar_type() == target_logits.scalar_type(),
              "spec_verify: draft_logits [B, k, V] of the target's dtype");
  TORCH_CHECK(draft_tokens.scalar_type() == at::kLong && draft_tokens.numel() == (long long)B * k,
              "spec_verify: draft_tokens int64 [B, k]");
  const c10::cuda::CUDAGuard guard(target_logits.device());
  auto tok = at::empty({B, k + 1}, target_logits.options().dtype(at::kLong));
  auto n = at::empty({B}, target_logits.options().dtype(at::kInt));
  auto lp = at::empty({B, k + 1}, target_logits.options().dtype(at::kFloat));
  if (B == 0) return {tok, n, lp};
  auto dt = draft_tokens.contiguous();
  RLB_DISPATCH_FLOAT(target_logits.scalar_type(), "spec_verify", [&] {
    spec::verify_kernel<scalar_t><<<B, spec::kThreads, 0, stream()>>>(
        (const scalar_t*)target_logits.data_ptr(), (const scalar_t*)draft_logits.data_ptr(),
        (const long long*)dt.data_ptr<int64_t>(), k, V, (float)temperature, (uint32_t)seed, (uint32_t)offset,
        (long long*)tok.data_ptr<int64_t>(), n.data_ptr<int>(), lp.data_ptr<float>());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {tok, n, lp};
}
