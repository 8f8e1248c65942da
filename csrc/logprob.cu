// Fused vocabulary reductions for RL losses.
//
// logprob_partials: one CTA per token row streams the (vocab-shard) logits once
// with 16-byte loads and keeps an online-softmax state per thread:
//   m = max(x/T),  s = sum exp(x/T - m),  u = sum (x/T) exp(x/T - m)
// merged across the CTA, plus the target logit x_t/T.  logprob = x_t/T - lse and
// entropy = lse - u/s follow on the host side (after a cross-shard combine when
// the vocabulary is tensor-parallel).
//
// logprob_bwd: dlogits = (dlogp / T) * (onehot(t) - exp(x/T - lse)), written in
// place over the logits (each element is read and written by the same thread).
#include "common.cuh"

namespace rlb {

struct SoftState {
  float m, s, u;
};

__device__ __forceinline__ SoftState merge(SoftState a, SoftState b) {
  if (a.m == -INFINITY) return b;
  if (b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  const float fa = __expf(a.m - m), fb = __expf(b.m - m);
  return {m, a.s * fa + b.s * fb, a.u * fa + b.u * fb};
}

__device__ __forceinline__ void push(SoftState& st, float x) {
  if (x > st.m) {
    const float f = __expf(st.m - x);
    st.s = st.s * f + 1.f;
    st.u = st.u * f + x;
    st.m = x;
  } else {
    const float e = __expf(x - st.m);
    st.s += e;
    st.u += x * e;
  }
}

// Push 8 values at once: one rescale per vector, one exp per element.
__device__ __forceinline__ void push8(SoftState& st, const float* f) {
  float mx = f[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) mx = fmaxf(mx, f[i]);
  if (mx > st.m) {
    const float r = __expf(st.m - mx);
    st.s *= r;
    st.u *= r;
    st.m = mx;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float e = __expf(f[i] - st.m);
    st.s += e;
    st.u += f[i] * e;
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
logprob_partials_kernel(const T* __restrict__ logits, const long long* __restrict__ targets, int V,
                        float inv_temp, float* __restrict__ m_out, float* __restrict__ s_out,
                        float* __restrict__ u_out, float* __restrict__ xt_out) {
  __shared__ SoftState red[32];
  const long long row = blockIdx.x;
  const T* x = logits + row * (long long)V;
  SoftState st{-INFINITY, 0.f, 0.f};
  if (sizeof(T) == 2 && V % 8 == 0) {
    const bf16x8* xv = reinterpret_cast<const bf16x8*>(x);
    for (int j = threadIdx.x; j < V / 8; j += blockDim.x) {
      float f[8];
      unpack8(xv[j], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] *= inv_temp;
      push8(st, f);
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) push(st, to_f(x[j]) * inv_temp);
  }
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    SoftState other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
                    __shfl_xor_sync(0xffffffffu, st.u, o)};
    st = merge(st, other);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) red[wid] = st;
  __syncthreads();
  if (wid == 0) {
    const int nw = blockDim.x >> 5;
    st = lane < nw ? red[lane] : SoftState{-INFINITY, 0.f, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      SoftState other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.s, o),
                      __shfl_xor_sync(0xffffffffu, st.u, o)};
      st = merge(st, other);
    }
    if (lane == 0) {
      m_out[row] = st.m;
      s_out[row] = st.s;
      u_out[row] = st.u;
      const long long t = targets[row];
      xt_out[row] = (t >= 0 && t < V) ? to_f(x[t]) * inv_temp : 0.f;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
logprob_bwd_kernel(const float* __restrict__ dlp, const T* logits, const long long* __restrict__ targets,
                   const float* __restrict__ lse, float inv_temp, int V, T* out) {
  const long long row = blockIdx.x;
  const float g = dlp[row];
  const float l = lse[row];
  const long long t = targets[row];
  const T* x = logits + row * (long long)V;
  T* o = out + row * (long long)V;
  const float gs = g * inv_temp;
  if (sizeof(T) == 2 && V % 8 == 0) {
    const bf16x8* xv = reinterpret_cast<const bf16x8*>(x);
    bf16x8* ov = reinterpret_cast<bf16x8*>(o);
    for (int j = threadIdx.x; j < V / 8; j += blockDim.x) {
      float f[8];
      unpack8(xv[j], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const long long col = (long long)j * 8 + i;
        f[i] = gs * ((col == t ? 1.f : 0.f) - __expf(f[i] * inv_temp - l));
      }
      ov[j] = pack8(f);
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const float p = __expf(to_f(x[j]) * inv_temp - l);
      o[j] = from_f<T>(gs * ((j == t ? 1.f : 0.f) - p));
    }
  }
}

}  // namespace rlb

using namespace rlb;

std::vector<at::Tensor> logprob_partials(at::Tensor logits, at::Tensor targets, double temperature) {
  RLB_CHECK(logits.is_cuda() && logits.dim() == 2 && logits.is_contiguous(), "logprob: logits must be [T, V]");
  const c10::cuda::CUDAGuard g(logits.device());
  const int T_ = logits.size(0), V = logits.size(1);
  auto tg = targets.to(at::kLong).contiguous();
  auto o = logits.options().dtype(at::kFloat);
  auto m = at::empty({T_}, o), s = at::empty({T_}, o), u = at::empty({T_}, o), xt = at::empty({T_}, o);
  if (T_ == 0) return {m, s, u, xt};
  RLB_DISPATCH_FLOAT(logits.scalar_type(), "logprob_partials", [&] {
    logprob_partials_kernel<scalar_t><<<T_, 256, 0, stream()>>>(
        (const scalar_t*)logits.data_ptr(), (long long*)tg.data_ptr<int64_t>(), V, (float)(1.0 / temperature),
        m.data_ptr<float>(), s.data_ptr<float>(), u.data_ptr<float>(), xt.data_ptr<float>());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {m, s, u, xt};
}

void logprob_bwd(at::Tensor dlp, at::Tensor logits, at::Tensor targets, at::Tensor lse, double temperature,
                 at::Tensor out) {
  RLB_CHECK(logits.is_contiguous() && out.is_contiguous() && out.sizes() == logits.sizes(), "logprob_bwd: layout");
  const c10::cuda::CUDAGuard g(logits.device());
  const int T_ = logits.size(0), V = logits.size(1);
  if (T_ == 0) return;
  auto tg = targets.to(at::kLong).contiguous();
  RLB_DISPATCH_FLOAT(logits.scalar_type(), "logprob_bwd", [&] {
    logprob_bwd_kernel<scalar_t><<<T_, 256, 0, stream()>>>(
        dlp.data_ptr<float>(), (const scalar_t*)logits.data_ptr(), (long long*)tg.data_ptr<int64_t>(), lse.data_ptr<float>(),
        (float)(1.0 / temperature), V, (scalar_t*)out.data_ptr());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
}
