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

// Unfiltered fast path: the vocabulary of each row is split over several CTAs
// (grid = splits x rows) so a decode batch of tens of rows still fills the GPU.
// Each CTA makes one pass over its slice (16-byte loads) keeping an online
// (max, sum-exp) pair and the running Gumbel argmax; a one-warp-per-row kernel
// merges the partials and reads back the chosen token's logit.
template <typename T>
__global__ void __launch_bounds__(256)
sample_partial_kernel(const T* __restrict__ logits, int V, int chunk, float inv_t, uint32_t seed,
                      const long long* __restrict__ offset_ptr, float4* __restrict__ parts) {
  __shared__ float red_m[8], red_s[8];
  __shared__ ArgMax red_am[8];
  const int row = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const T* x = logits + (long long)row * V;
  const long long off = *offset_ptr;
  const uint32_t stream_id = (uint32_t)row * 0x632BE5ABu + (uint32_t)off * 0x9E3779B1u + (uint32_t)(off >> 32);
  const int beg = split * chunk, end = min(V, beg + chunk);
  float m = -INFINITY, s = 0.f;
  ArgMax best{-INFINITY, 0x7fffffff};
  auto push = [&](float v, int j) {
    if (v > m) {
      s = s * __expf(m - v) + 1.f;
      m = v;
    } else {
      s += __expf(v - m);
    }
    const float u = uniform01(seed, stream_id, (uint32_t)j);
    best = amax(best, ArgMax{v - __logf(-__logf(u)), j});
  };
  if (sizeof(T) == 2 && (beg % 8) == 0 && (V % 8) == 0) {
    const bf16x8* xv = reinterpret_cast<const bf16x8*>(x);
    for (int jv = beg / 8 + threadIdx.x; jv < (end + 7) / 8; jv += blockDim.x) {
      float f[8];
      unpack8(xv[jv], f);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (jv * 8 + i < end) push(f[i] * inv_t, jv * 8 + i);
    }
  } else {
    for (int j = beg + threadIdx.x; j < end; j += blockDim.x) push(to_f(x[j]) * inv_t, j);
  }
  // merge within the warp
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
    ArgMax other{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
    best = amax(best, other);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    red_m[wid] = m;
    red_s[wid] = s;
    red_am[wid] = best;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY, Ssum = 0.f;
    ArgMax B{-INFINITY, 0x7fffffff};
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) M = fmaxf(M, red_m[k]);
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) {
      if (red_m[k] != -INFINITY) Ssum += red_s[k] * __expf(red_m[k] - M);
      B = amax(B, red_am[k]);
    }
    parts[(long long)row * S + split] = make_float4(M, Ssum, B.key, __int_as_float(B.idx));
  }
}

template <typename T>
__global__ void sample_combine_kernel(const T* __restrict__ logits, const float4* __restrict__ parts, int S, int V,
                                     float inv_t, long long* __restrict__ out_tok, float* __restrict__ out_lp,
                                     int rows) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float m = -INFINITY, s = 0.f;
  ArgMax best{-INFINITY, 0x7fffffff};
  for (int k = lane; k < S; k += 32) {
    const float4 p = parts[(long long)row * S + k];
    const float mm = fmaxf(m, p.x);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (p.x == -INFINITY ? 0.f : p.y * __expf(p.x - mm));
    m = mm;
    best = amax(best, ArgMax{p.z, __float_as_int(p.w)});
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
    ArgMax other{__shfl_xor_sync(0xffffffffu, best.key, o), __shfl_xor_sync(0xffffffffu, best.idx, o)};
    best = amax(best, other);
  }
  if (lane == 0) {
    const int tok = (best.idx >= 0 && best.idx < V) ? best.idx : 0;
    out_tok[row] = tok;
    out_lp[row] = to_f(logits[(long long)row * V + tok]) * inv_t - (m + __logf(s));
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
  const bool unfiltered = (top_k <= 0 || top_k >= V) && top_p >= 1.0;
  if (unfiltered) {
    int S = std::max(1, std::min((2 * num_sms() + B - 1) / B, V / 4096));
    const int chunk = ((V + S - 1) / S + 7) / 8 * 8;
    S = (V + chunk - 1) / chunk;
    auto parts = at::empty({(long long)B * S * 4}, logits.options().dtype(at::kFloat));
    RLB_DISPATCH_FLOAT(logits.scalar_type(), "sample", [&] {
      sample_partial_kernel<scalar_t><<<dim3(S, B), 256, 0, stream()>>>(
          (const scalar_t*)logits.data_ptr(), V, chunk, inv_t, (uint32_t)(seed & 0xffffffff),
          (long long*)offset.data_ptr<int64_t>(), reinterpret_cast<float4*>(parts.data_ptr<float>()));
      sample_combine_kernel<scalar_t><<<(B + 7) / 8, 256, 0, stream()>>>(
          (const scalar_t*)logits.data_ptr(), reinterpret_cast<const float4*>(parts.data_ptr<float>()), S, V, inv_t,
          (long long*)out_tok.data_ptr<int64_t>(), out_lp.data_ptr<float>(), B);
    });
    RLB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  RLB_DISPATCH_FLOAT(logits.scalar_type(), "sample", [&] {
    sample_kernel<scalar_t><<<B, 256, 0, stream()>>>((const scalar_t*)logits.data_ptr(), V, inv_t, (int)top_k,
                                                      (float)top_p, (uint32_t)(seed & 0xffffffff),
                                                      (long long*)offset.data_ptr<int64_t>(), (long long*)out_tok.data_ptr<int64_t>(),
                                                      out_lp.data_ptr<float>());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
}
