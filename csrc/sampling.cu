// Token sampling: temperature, top-k, top-p, Gumbel-max draw and the sampled
// token's log-probability under the processed distribution.
//
// One CTA per row.  Without filtering the kernel makes ONE pass over the row:
// an online softmax (max, sum-exp) and a running argmax of x/T + g_i where
// g_i = -log(-log(u_i)) is Gumbel noise from a counter-based hash of
// (seed, row, step, i) - an exact draw from softmax(x/T).
// With top-k / top-p the kept set {x >= tau} is found by bisection on tau
// (count >= k, then mass >= p over the top-k set), then the same draw runs over
// the kept set.  The random step offset is read from device memory so a
// captured decode graph advances it between replays.
#include "common.cuh"

namespace rlb {

struct ArgMax {
  float key;
  int idx;
};

__device__ __forceinline__ ArgMax amax(ArgMax a, ArgMax b) {
  if (b.key > a.key || (b.key == a.key && b.idx < a.idx)) return b;
  return a;
}

template <typename T>
__device__ __forceinline__ float ld(const T* x, int j, float inv_t) {
  return to_f(x[j]) * inv_t;
}

template <typename T>
__global__ void __launch_bounds__(256)
sample_kernel(const T* __restrict__ logits, int V, float inv_t, int top_k, float top_p, uint32_t seed,
              const long long* __restrict__ offset_ptr, long long* __restrict__ out_tok,
              float* __restrict__ out_lp) {
  __shared__ float red[32];
  __shared__ ArgMax red_am[32];
  const int row = blockIdx.x;
  const T* x = logits + (long long)row * V;
  const long long off = *offset_ptr;
  const uint32_t stream_id = (uint32_t)row * 0x632BE5ABu + (uint32_t)off * 0x9E3779B1u + (uint32_t)(off >> 32);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;

  // ---- row max / min ----
  float mx = -INFINITY, mn = INFINITY;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = ld(x, j, inv_t);
    mx = fmaxf(mx, v);
    mn = fminf(mn, v);
  }
  mx = block_max(mx, red);
  mn = -block_max(-mn, red);

  float tau = -INFINITY;
  const bool filt_k = top_k > 0 && top_k < V;
  const bool filt_p = top_p < 1.f;
  if (filt_k) {
    float lo = mn, hi = mx;  // invariant: count(x >= lo) >= k
    for (int it = 0; it < 28; ++it) {
      const float mid = 0.5f * (lo + hi);
      float c = 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x) c += ld(x, j, inv_t) >= mid ? 1.f : 0.f;
      c = block_sum(c, red);
      if (c >= (float)top_k) lo = mid; else hi = mid;
    }
    tau = lo;
  }
  if (filt_p) {
    float z = 0.f;
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const float v = ld(x, j, inv_t);
      if (v >= tau) z += __expf(v - mx);
    }
    z = block_sum(z, red);
    float lo = fmaxf(tau, mn), hi = mx;  // invariant: mass(x >= lo) >= p
    for (int it = 0; it < 28; ++it) {
      const float mid = 0.5f * (lo + hi);
      float s = 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float v = ld(x, j, inv_t);
        if (v >= mid) s += __expf(v - mx);
      }
      s = block_sum(s, red);
      if (s >= top_p * z) lo = mid; else hi = mid;
    }
    tau = fmaxf(tau, lo);
  }

  // ---- kept-set sum-exp and Gumbel argmax ----
  float se = 0.f;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float v = ld(x, j, inv_t);
    if (v < tau) continue;
    se += __expf(v - mx);
    const float u = uniform01(seed, stream_id, (uint32_t)j);
    const float key = v - __logf(-__logf(u));
    best = amax(best, ArgMax{key, j});
  }
  se = block_sum(se, red);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax other{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
    best = amax(best, other);
  }
  __syncthreads();
  if (lane == 0) red_am[wid] = best;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? red_am[lane] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax other{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
      best = amax(best, other);
    }
    if (lane == 0) {
      const int tok = best.idx < V ? best.idx : 0;
      out_tok[row] = tok;
      out_lp[row] = ld(x, tok, inv_t) - (mx + __logf(se));
    }
  }
}

}  // namespace rlb

using namespace rlb;

void sample(at::Tensor logits, double temperature, int64_t top_k, double top_p, int64_t seed, at::Tensor offset,
            at::Tensor out_tok, at::Tensor out_lp) {
  RLB_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "sample: logits must be [B, V]");
  RLB_CHECK(offset.scalar_type() == at::kLong && offset.is_cuda(), "sample: offset must be a CUDA int64 tensor");
  RLB_CHECK(out_tok.scalar_type() == at::kLong && out_lp.scalar_type() == at::kFloat, "sample: output dtypes");
  const c10::cuda::CUDAGuard g(logits.device());
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  const float inv_t = (float)(1.0 / std::max(temperature, 1e-6));
  RLB_DISPATCH_FLOAT(logits.scalar_type(), "sample", [&] {
    sample_kernel<scalar_t><<<B, 256, 0, stream()>>>((const scalar_t*)logits.data_ptr(), V, inv_t, (int)top_k,
                                                      (float)top_p, (uint32_t)(seed & 0xffffffff),
                                                      (long long*)offset.data_ptr<int64_t>(), (long long*)out_tok.data_ptr<int64_t>(),
                                                      out_lp.data_ptr<float>());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
}
