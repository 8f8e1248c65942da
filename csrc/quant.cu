// Block-scaled e4m3 quantisation.
//
// quant_fp8_block: one CTA per 128x128 weight block: block amax -> scale =
// amax / 448 (optionally rounded UP to a power of two by exponent-bit
// arithmetic, no libm) -> saturating e4m3 cast.  Scales are fp32
// [ceil(N/128), ceil(K/128)].
// quant_fp8_group: one warp per 1 x group activation slice, same scale rule,
// scales fp32 [T, K/group] (row-major).
#include "common.cuh"

namespace rlb {

constexpr float kFp8Max = 448.f;

// Smallest power of two >= s (s > 0, finite): bump the exponent when any
// mantissa bit is set.
__device__ __forceinline__ float pow2_ceil(float s) {
  uint32_t b = __float_as_uint(s);
  if (b & 0x007fffffu) {
    b = (b & 0xff800000u) + 0x00800000u;
  }
  return __uint_as_float(b & 0xff800000u);
}

__device__ __forceinline__ float fp8_scale(float amax, bool pow2) {
  float s = fmaxf(amax, 1e-12f) / kFp8Max;
  return pow2 ? pow2_ceil(s) : s;
}

template <typename T>
__global__ void __launch_bounds__(256)
quant_block_kernel(const T* __restrict__ w, __nv_fp8_e4m3* __restrict__ q, float* __restrict__ scales, int N, int K,
                   int blk, bool pow2) {
  __shared__ float red[32];
  const int bn = blockIdx.y, bk = blockIdx.x;
  const int kb = gridDim.x;
  const int r0 = bn * blk, c0 = bk * blk;
  float amax = 0.f;
  for (int e = threadIdx.x; e < blk * blk; e += blockDim.x) {
    const int r = r0 + e / blk, c = c0 + e % blk;
    if (r < N && c < K) amax = fmaxf(amax, fabsf(to_f(w[(size_t)r * K + c])));
  }
  amax = block_max(amax, red);
  const float s = fp8_scale(amax, pow2);
  const float inv = 1.f / s;
  if (threadIdx.x == 0) scales[bn * kb + bk] = s;
  for (int e = threadIdx.x; e < blk * blk; e += blockDim.x) {
    const int r = r0 + e / blk, c = c0 + e % blk;
    if (r < N && c < K) {
      const float v = fminf(fmaxf(to_f(w[(size_t)r * K + c]) * inv, -kFp8Max), kFp8Max);
      q[(size_t)r * K + c] = __nv_fp8_e4m3(v);
    }
  }
}

template <typename T>
__global__ void quant_group_kernel(const T* __restrict__ x, __nv_fp8_e4m3* __restrict__ q, float* __restrict__ scales,
                                   long long groups_total, int K, int group, bool pow2) {
  const int lane = threadIdx.x & 31;
  const long long gi = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gi >= groups_total) return;
  const int gpr = K / group;
  const long long row = gi / gpr;
  const int gc = gi % gpr;
  const T* src = x + row * K + (long long)gc * group;
  float amax = 0.f;
  for (int j = lane; j < group; j += 32) amax = fmaxf(amax, fabsf(to_f(src[j])));
  amax = warp_max(amax);
  const float s = fp8_scale(amax, pow2);
  const float inv = 1.f / s;
  if (lane == 0) scales[gi] = s;
  __nv_fp8_e4m3* dst = q + row * K + (long long)gc * group;
  for (int j = lane; j < group; j += 32) dst[j] = __nv_fp8_e4m3(fminf(fmaxf(to_f(src[j]) * inv, -kFp8Max), kFp8Max));
}

// Same quantisation; the scale of (row, group g) goes to s_t[g * Mp + row]
// (MN-major, the layout the block-scaled GEMM fetches per K block).
template <typename T>
__global__ void quant_group_t_kernel(const T* __restrict__ x, __nv_fp8_e4m3* __restrict__ q, float* __restrict__ s_t,
                                     long long groups_total, int K, int group, int Mp, bool pow2) {
  const int lane = threadIdx.x & 31;
  const long long gi = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gi >= groups_total) return;
  const int gpr = K / group;
  const long long row = gi / gpr;
  const int gc = gi % gpr;
  const T* src = x + row * K + (long long)gc * group;
  float amax = 0.f;
  for (int j = lane; j < group; j += 32) amax = fmaxf(amax, fabsf(to_f(src[j])));
  amax = warp_max(amax);
  const float s = fp8_scale(amax, pow2);
  const float inv = 1.f / s;
  if (lane == 0) s_t[(long long)gc * Mp + row] = s;
  __nv_fp8_e4m3* dst = q + row * K + (long long)gc * group;
  for (int j = lane; j < group; j += 32) dst[j] = __nv_fp8_e4m3(fminf(fmaxf(to_f(src[j]) * inv, -kFp8Max), kFp8Max));
}

}  // namespace rlb

using namespace rlb;

std::vector<at::Tensor> quant_fp8_block(at::Tensor w, int64_t blk, bool pow2, c10::optional<at::Tensor> out,
                                        c10::optional<at::Tensor> out_scale) {
  RLB_CHECK(w.is_cuda() && w.dim() == 2 && w.is_contiguous(), "quant_fp8_block: 2-D contiguous CUDA weight expected");
  const c10::cuda::CUDAGuard g(w.device());
  const int N = w.size(0), K = w.size(1);
  const int nb = (N + blk - 1) / blk, kb = (K + blk - 1) / blk;
  at::Tensor q = (out.has_value() && out->defined()) ? *out : at::empty({N, K}, w.options().dtype(at::kFloat8_e4m3fn));
  at::Tensor s = (out_scale.has_value() && out_scale->defined()) ? *out_scale
                                                                    : at::empty({nb, kb}, w.options().dtype(at::kFloat));
  RLB_CHECK(q.scalar_type() == at::kFloat8_e4m3fn && q.numel() == (long long)N * K, "quant_fp8_block: bad out");
  RLB_CHECK(s.numel() == (long long)nb * kb, "quant_fp8_block: bad scale out");
  if (N == 0 || K == 0) return {q, s};
  dim3 grid(kb, nb);
  RLB_DISPATCH_FLOAT(w.scalar_type(), "quant_fp8_block", [&] {
    quant_block_kernel<scalar_t><<<grid, 256, 0, stream()>>>((const scalar_t*)w.data_ptr(),
                                                              (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>(), N, K,
                                                              (int)blk, pow2);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {q, s};
}

std::vector<at::Tensor> quant_fp8_group(at::Tensor x, int64_t group, bool pow2) {
  RLB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "quant_fp8_group: 2-D contiguous CUDA input expected");
  RLB_CHECK(x.size(1) % group == 0, "quant_fp8_group: K must be a multiple of the group size");
  const c10::cuda::CUDAGuard g(x.device());
  const long long T_ = x.size(0);
  const int K = x.size(1);
  auto q = at::empty({T_, K}, x.options().dtype(at::kFloat8_e4m3fn));
  auto s = at::empty({T_, K / group}, x.options().dtype(at::kFloat));
  const long long groups = T_ * (K / group);
  if (groups == 0) return {q, s};
  const int warps = 8;
  RLB_DISPATCH_FLOAT(x.scalar_type(), "quant_fp8_group", [&] {
    quant_group_kernel<scalar_t><<<(groups + warps - 1) / warps, warps * 32, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>(), groups, K, (int)group,
        pow2);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {q, s};
}

// (q [T, K] e4m3, s_t [K/group, Mp] fp32) with Mp = T rounded up to 128 (pad scales 1.0)
std::vector<at::Tensor> quant_fp8_group_t(at::Tensor x, int64_t group, bool pow2) {
  RLB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "quant_fp8_group_t: 2-D contiguous CUDA input expected");
  RLB_CHECK(x.size(1) % group == 0, "quant_fp8_group_t: K must be a multiple of the group size");
  const c10::cuda::CUDAGuard g(x.device());
  const long long T_ = x.size(0);
  const int K = x.size(1);
  const int Mp = (int)((T_ + 127) / 128 * 128);
  auto q = at::empty({T_, K}, x.options().dtype(at::kFloat8_e4m3fn));
  auto s = at::ones({K / group, (long long)std::max(Mp, 128)}, x.options().dtype(at::kFloat));
  const long long groups = T_ * (K / group);
  if (groups == 0) return {q, s};
  const int warps = 8;
  RLB_DISPATCH_FLOAT(x.scalar_type(), "quant_fp8_group_t", [&] {
    quant_group_t_kernel<scalar_t><<<(groups + warps - 1) / warps, warps * 32, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), (__nv_fp8_e4m3*)q.data_ptr(), s.data_ptr<float>(), groups, K, (int)group,
        (int)s.size(1), pow2);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {q, s};
}
