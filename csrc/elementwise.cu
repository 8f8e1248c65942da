// Element-wise fused ops: RoPE over packed QKV, SwiGLU forward/backward,
// paged KV-cache writes.
//
// RoPE: rotate_half convention with a precomputed fp32 [max_pos, hd] table
// (first half cos, second half sin).  One thread handles 4 rotation pairs of
// one head; v heads are copied.  ``inverse`` rotates by -theta (the backward).
//
// SwiGLU: out = silu(gate) * up on gu = [T, 2F] (gate | up); 8 elements per
// thread with 16-byte accesses for bf16.
#include "common.cuh"

namespace rlb {

template <typename T>
__global__ void rope_qkv_kernel(const T* __restrict__ in, T* __restrict__ out, const int* __restrict__ pos,
                                const float* __restrict__ cache, int T_, int nq, int nkv, int hd, int inverse) {
  const int half = hd / 2;
  const int quads = half / 4;  // 4 pairs per thread
  const int heads = nq + 2 * nkv;
  const long long total = (long long)T_ * heads * quads;
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
       id += (long long)gridDim.x * blockDim.x) {
    const int q = id % quads;
    const long long th = id / quads;
    const int h = th % heads;
    const int t = th / heads;
    const size_t base = ((size_t)t * heads + h) * hd;
    const int i0 = q * 4;
    if (h >= nq + nkv) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        out[base + i0 + k] = in[base + i0 + k];
        out[base + half + i0 + k] = in[base + half + i0 + k];
      }
      continue;
    }
    const float* cs = cache + (size_t)pos[t] * hd;
    const float sgn = inverse ? -1.f : 1.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float c = cs[i0 + k];
      const float s = sgn * cs[half + i0 + k];
      const float x1 = to_f(in[base + i0 + k]);
      const float x2 = to_f(in[base + half + i0 + k]);
      out[base + i0 + k] = from_f<T>(x1 * c - x2 * s);
      out[base + half + i0 + k] = from_f<T>(x2 * c + x1 * s);
    }
  }
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ out, long long rows, int F) {
  pdl_launch_dependents();
  const bool vec = (sizeof(T) == 2) && (F % 8 == 0);
  if (vec) {
    const int fv = F / 8;
    const long long total = rows * fv;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
         id += (long long)gridDim.x * blockDim.x) {
      const long long r = id / fv;
      const int j = id % fv;
      const bf16x8* g = reinterpret_cast<const bf16x8*>(gu + r * 2 * F);
      float a[8], b[8];
      unpack8(g[j], a);
      unpack8(g[fv + j], b);
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = silu_f(a[i]) * b[i];
      reinterpret_cast<bf16x8*>(out + r * F)[j] = pack8(a);
    }
  } else {
    const long long total = rows * F;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
         id += (long long)gridDim.x * blockDim.x) {
      const long long r = id / F;
      const int j = id % F;
      const float g = to_f(gu[r * 2 * F + j]), u = to_f(gu[r * 2 * F + F + j]);
      out[r * F + j] = from_f<T>(silu_f(g) * u);
    }
  }
}

// d gate = dout * up * sig * (1 + g * (1 - sig)),  d up = dout * silu(g)
template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ dout, const T* __restrict__ gu, T* __restrict__ dgu,
                                  long long rows, int F) {
  const bool vec = (sizeof(T) == 2) && (F % 8 == 0);
  if (vec) {
    const int fv = F / 8;
    const long long total = rows * fv;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
         id += (long long)gridDim.x * blockDim.x) {
      const long long r = id / fv;
      const int j = id % fv;
      const bf16x8* g = reinterpret_cast<const bf16x8*>(gu + r * 2 * F);
      float a[8], b[8], d[8], da[8], db[8];
      unpack8(g[j], a);
      unpack8(g[fv + j], b);
      unpack8(reinterpret_cast<const bf16x8*>(dout + r * F)[j], d);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float sg = 1.f / (1.f + __expf(-a[i]));
        da[i] = d[i] * b[i] * sg * (1.f + a[i] * (1.f - sg));
        db[i] = d[i] * a[i] * sg;
      }
      bf16x8* o = reinterpret_cast<bf16x8*>(dgu + r * 2 * F);
      o[j] = pack8(da);
      o[fv + j] = pack8(db);
    }
  } else {
    const long long total = rows * F;
    for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
         id += (long long)gridDim.x * blockDim.x) {
      const long long r = id / F;
      const int j = id % F;
      const float g = to_f(gu[r * 2 * F + j]), u = to_f(gu[r * 2 * F + F + j]);
      const float d = to_f(dout[r * F + j]);
      const float sg = 1.f / (1.f + __expf(-g));
      dgu[r * 2 * F + j] = from_f<T>(d * u * sg * (1.f + g * (1.f - sg)));
      dgu[r * 2 * F + F + j] = from_f<T>(d * g * sg);
    }
  }
}

// k, v: [T, nkv, hd] with row stride `src_stride` elements (views of the QKV buffer).
// caches: [num_blocks * block_size, nkv, hd] contiguous.  Optional fp8 caches
// are written with a per-tensor inverse scale.
template <typename T, typename C>
__global__ void write_kv_kernel(const T* __restrict__ k, const T* __restrict__ v, long long k_stride,
                                long long v_stride, C* __restrict__ kc, C* __restrict__ vc,
                                const long long* __restrict__ slots, int T_, int row_elems, float inv_k,
                                float inv_v, long long n_slots) {
  const long long total = (long long)T_ * row_elems;
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
       id += (long long)gridDim.x * blockDim.x) {
    const int t = id / row_elems;
    const int e = id % row_elems;
    const long long slot = slots[t];
    if (slot < 0 || !RLB_IN_BOUNDS(slot, n_slots, kBoundsKvSlot)) continue;
    const float kv = to_f(k[t * k_stride + e]) * inv_k;
    const float vv = to_f(v[t * v_stride + e]) * inv_v;
    if constexpr (std::is_same<C, __nv_fp8_e4m3>::value) {
      kc[slot * row_elems + e] = __nv_fp8_e4m3(kv);
      vc[slot * row_elems + e] = __nv_fp8_e4m3(vv);
    } else {
      kc[slot * row_elems + e] = from_f<C>(kv);
      vc[slot * row_elems + e] = from_f<C>(vv);
    }
  }
}

inline int ew_grid(long long total, int threads = 256) {
  long long b = (total + threads - 1) / threads;
  long long cap = (long long)num_sms() * 16;
  return (int)std::max<long long>(1, std::min(b, cap));
}

}  // namespace rlb

using namespace rlb;

at::Tensor rope_qkv(at::Tensor qkv, at::Tensor positions, at::Tensor cache, int64_t nq, int64_t nkv, int64_t hd,
                    bool inverse) {
  RLB_CHECK(qkv.is_cuda() && qkv.is_contiguous() && qkv.dim() == 2, "rope: qkv must be contiguous [T, (nq+2nkv)*hd]");
  RLB_CHECK(qkv.size(1) == (nq + 2 * nkv) * hd, "rope: qkv width mismatch");
  RLB_CHECK(hd % 8 == 0, "rope: head_dim must be a multiple of 8");
  RLB_CHECK(cache.scalar_type() == at::kFloat && cache.size(1) == hd, "rope: cache must be fp32 [max_pos, hd]");
  const c10::cuda::CUDAGuard g(qkv.device());
  auto pos = positions.to(at::kInt).contiguous();
  auto out = at::empty_like(qkv);
  const int T_ = qkv.size(0);
  if (T_ == 0) return out;
  long long total = (long long)T_ * (nq + 2 * nkv) * (hd / 8);
  RLB_DISPATCH_FLOAT(qkv.scalar_type(), "rope_qkv", [&] {
    rope_qkv_kernel<scalar_t><<<ew_grid(total), 256, 0, stream()>>>(
        (const scalar_t*)qkv.data_ptr(), (scalar_t*)out.data_ptr(), pos.data_ptr<int>(), cache.data_ptr<float>(), T_,
        (int)nq, (int)nkv, (int)hd, inverse ? 1 : 0);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return out;
}

at::Tensor swiglu_fwd(at::Tensor gu) {
  RLB_CHECK(gu.is_cuda() && gu.is_contiguous() && gu.size(-1) % 2 == 0, "swiglu: bad input");
  const c10::cuda::CUDAGuard g(gu.device());
  const int F = gu.size(-1) / 2;
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto out = at::empty(sizes, gu.options());
  const long long rows = gu.numel() / (2 * F);
  if (rows == 0) return out;
  RLB_DISPATCH_FLOAT(gu.scalar_type(), "swiglu_fwd", [&] {
    swiglu_fwd_kernel<scalar_t><<<ew_grid(rows * F / 8 + 1), 256, 0, stream()>>>(
        (const scalar_t*)gu.data_ptr(), (scalar_t*)out.data_ptr(), rows, F);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return out;
}

at::Tensor swiglu_bwd(at::Tensor dout, at::Tensor gu) {
  RLB_CHECK(gu.is_cuda() && gu.is_contiguous() && dout.is_contiguous(), "swiglu_bwd: bad input");
  const c10::cuda::CUDAGuard g(gu.device());
  const int F = gu.size(-1) / 2;
  auto dgu = at::empty_like(gu);
  const long long rows = gu.numel() / (2 * F);
  if (rows == 0) return dgu;
  RLB_DISPATCH_FLOAT(gu.scalar_type(), "swiglu_bwd", [&] {
    swiglu_bwd_kernel<scalar_t><<<ew_grid(rows * F / 8 + 1), 256, 0, stream()>>>(
        (const scalar_t*)dout.data_ptr(), (const scalar_t*)gu.data_ptr(), (scalar_t*)dgu.data_ptr(), rows, F);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return dgu;
}

// fp8 caches store k / k_scale and v / v_scale (per-tensor scales of the layer).
void write_kv_cache(at::Tensor k, at::Tensor v, at::Tensor k_cache, at::Tensor v_cache, at::Tensor slots,
                    double k_scale, double v_scale) {
  RLB_CHECK(k.dim() == 3 && v.dim() == 3, "write_kv_cache: k/v must be [T, nkv, hd]");
  RLB_CHECK(k.stride(2) == 1 && k.stride(1) == k.size(2) && v.stride(2) == 1 && v.stride(1) == v.size(2),
            "write_kv_cache: heads must be contiguous within a token");
  RLB_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "write_kv_cache: caches must be contiguous");
  const c10::cuda::CUDAGuard g(k.device());
  const int T_ = k.size(0);
  if (T_ == 0) return;
  const int row = k.size(1) * k.size(2);
  auto sl = slots.to(at::kLong).contiguous();
  long long total = (long long)T_ * row;
  const long long n_slots = std::min(k_cache.numel(), v_cache.numel()) / row;
  RLB_DISPATCH_FLOAT(k.scalar_type(), "write_kv_cache", [&] {
    if (k_cache.scalar_type() == at::kFloat8_e4m3fn) {
      write_kv_kernel<scalar_t, __nv_fp8_e4m3><<<ew_grid(total), 256, 0, stream()>>>(
          (const scalar_t*)k.data_ptr(), (const scalar_t*)v.data_ptr(), k.stride(0), v.stride(0),
          (__nv_fp8_e4m3*)k_cache.data_ptr(), (__nv_fp8_e4m3*)v_cache.data_ptr(), (long long*)sl.data_ptr<int64_t>(), T_,
          row, (float)(1.0 / k_scale), (float)(1.0 / v_scale), n_slots);
    } else {
      RLB_CHECK(k_cache.scalar_type() == k.scalar_type(), "write_kv_cache: cache dtype mismatch");
      write_kv_kernel<scalar_t, scalar_t><<<ew_grid(total), 256, 0, stream()>>>(
          (const scalar_t*)k.data_ptr(), (const scalar_t*)v.data_ptr(), k.stride(0), v.stride(0),
          (scalar_t*)k_cache.data_ptr(), (scalar_t*)v_cache.data_ptr(), (long long*)sl.data_ptr<int64_t>(), T_, row, 1.f, 1.f, n_slots);
    }
  });
  RLB_CUDA_CHECK(cudaGetLastError());
}

int64_t bounds_error_elementwise(bool reset) { return rlb::rlb_bounds_error(reset); }
