// Fused AdamW over flat fp32 buffers + deterministic sum of squares.
//
// adamw_step: one launch updates master weights, both moments and (optionally)
// writes the bf16 working copy of the parameters; 4 elements per thread with
// 16-byte accesses.  Bias corrections are folded into two host-computed scalars.
#include "common.cuh"

namespace rlb {

template <typename G>
__global__ void adamw_kernel(float* __restrict__ p, const G* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ out, long long n, float lr, float b1,
                             float b2, float eps, float wd, float step_size, float inv_bc2_sqrt, float gscale) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float gg[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) gg[k] = to_f(g[i * 4 + k]) * gscale;
    float* P = &pp.x;
    float* M = &mm.x;
    float* Vv = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      M[k] = b1 * M[k] + (1.f - b1) * gg[k];
      Vv[k] = b2 * Vv[k] + (1.f - b2) * gg[k] * gg[k];
      const float denom = sqrtf(Vv[k]) * inv_bc2_sqrt + eps;
      P[k] = P[k] * (1.f - lr * wd) - step_size * M[k] / denom;
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (out) {
      __nv_bfloat162 a = __floats2bfloat162_rn(P[0], P[1]);
      __nv_bfloat162 b = __floats2bfloat162_rn(P[2], P[3]);
      uint2 packed;
      packed.x = *reinterpret_cast<uint32_t*>(&a);
      packed.y = *reinterpret_cast<uint32_t*>(&b);
      reinterpret_cast<uint2*>(out)[i] = packed;
    }
  }
  // tail
  const long long t0 = n4 * 4;
  for (long long i = t0 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gg = to_f(g[i]) * gscale;
    m[i] = b1 * m[i] + (1.f - b1) * gg;
    v[i] = b2 * v[i] + (1.f - b2) * gg * gg;
    p[i] = p[i] * (1.f - lr * wd) - step_size * m[i] / (sqrtf(v[i]) * inv_bc2_sqrt + eps);
    if (out) out[i] = __float2bfloat16_rn(p[i]);
  }
}

template <typename T>
__global__ void sumsq_partial_kernel(const T* __restrict__ x, long long n, float* __restrict__ part) {
  __shared__ float red[32];
  float s = 0.f;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = to_f(x[i]);
    s += v * v;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void sum_partials_kernel(const float* __restrict__ part, int n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += part[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[0] = s;
}

}  // namespace rlb

using namespace rlb;

void adamw_step(at::Tensor master, at::Tensor grad, at::Tensor exp_avg, at::Tensor exp_avg_sq,
                c10::optional<at::Tensor> param_out, double lr, double beta1, double beta2, double eps,
                double weight_decay, int64_t step, double grad_scale) {
  RLB_CHECK(master.scalar_type() == at::kFloat && exp_avg.scalar_type() == at::kFloat &&
                exp_avg_sq.scalar_type() == at::kFloat,
            "adamw: master/moments must be fp32");
  RLB_CHECK(master.is_contiguous() && grad.is_contiguous() && exp_avg.is_contiguous() && exp_avg_sq.is_contiguous(),
            "adamw: buffers must be contiguous");
  const long long n = master.numel();
  RLB_CHECK(grad.numel() == n && exp_avg.numel() == n && exp_avg_sq.numel() == n, "adamw: size mismatch");
  RLB_CHECK(reinterpret_cast<uintptr_t>(master.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(exp_avg.data_ptr()) % 16 == 0 &&
                reinterpret_cast<uintptr_t>(exp_avg_sq.data_ptr()) % 16 == 0,
            "adamw: buffers must be 16-byte aligned");
  __nv_bfloat16* out = nullptr;
  if (param_out.has_value() && param_out->defined()) {
    RLB_CHECK(param_out->scalar_type() == at::kBFloat16 && param_out->numel() == n && param_out->is_contiguous(),
              "adamw: param_out must be contiguous bf16 of the same length");
    RLB_CHECK(reinterpret_cast<uintptr_t>(param_out->data_ptr()) % 8 == 0, "adamw: param_out must be 8-byte aligned");
    out = (__nv_bfloat16*)param_out->data_ptr();
  }
  if (n == 0) return;
  const c10::cuda::CUDAGuard g(master.device());
  const double bc1 = 1.0 - std::pow(beta1, (double)step);
  const double bc2 = 1.0 - std::pow(beta2, (double)step);
  const float step_size = (float)(lr / bc1);
  const float inv_bc2_sqrt = (float)(1.0 / std::sqrt(bc2));
  const int threads = 256;
  const int blocks = (int)std::min<long long>((n / 4 + threads - 1) / threads + 1, (long long)num_sms() * 8);
  if (grad.scalar_type() == at::kFloat) {
    adamw_kernel<float><<<blocks, threads, 0, stream()>>>(
        master.data_ptr<float>(), grad.data_ptr<float>(), exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(), out,
        n, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)weight_decay, step_size, inv_bc2_sqrt,
        (float)grad_scale);
  } else {
    RLB_CHECK(grad.scalar_type() == at::kBFloat16, "adamw: grad must be fp32 or bf16");
    adamw_kernel<__nv_bfloat16><<<blocks, threads, 0, stream()>>>(
        master.data_ptr<float>(), (const __nv_bfloat16*)grad.data_ptr(), exp_avg.data_ptr<float>(),
        exp_avg_sq.data_ptr<float>(), out, n, (float)lr, (float)beta1, (float)beta2, (float)eps, (float)weight_decay,
        step_size, inv_bc2_sqrt, (float)grad_scale);
  }
  RLB_CUDA_CHECK(cudaGetLastError());
}

at::Tensor sum_sq(at::Tensor x) {
  RLB_CHECK(x.is_cuda() && x.is_contiguous(), "sum_sq: contiguous CUDA tensor expected");
  const c10::cuda::CUDAGuard g(x.device());
  auto out = at::zeros({}, x.options().dtype(at::kFloat));
  const long long n = x.numel();
  if (n == 0) return out;
  const int blocks = (int)std::min<long long>((n + 255) / 256, (long long)num_sms() * 4);
  auto part = at::empty({blocks}, x.options().dtype(at::kFloat));
  RLB_DISPATCH_FLOAT(x.scalar_type(), "sum_sq", [&] {
    sumsq_partial_kernel<scalar_t><<<blocks, 256, 0, stream()>>>((const scalar_t*)x.data_ptr(), n,
                                                                  part.data_ptr<float>());
  });
  sum_partials_kernel<<<1, 256, 0, stream()>>>(part.data_ptr<float>(), blocks, out.data_ptr<float>());
  RLB_CUDA_CHECK(cudaGetLastError());
  return out;
}
