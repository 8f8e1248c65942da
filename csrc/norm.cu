// RMSNorm forward / backward and the fused residual-add + RMSNorm.
//
// One warp per row (rows are hidden vectors of a packed token batch).  The
// forward makes two passes over the row (sum of squares, then normalise); the
// second pass re-reads from L1, so DRAM sees one read of x (and delta) and
// one write of y (and the residual sum).  bf16 rows with H % 8 == 0 use 16-byte
// vector accesses.  The backward accumulates the weight gradient per warp in
// shared memory and writes one fp32 partial row per CTA; a second kernel sums
// the partials (deterministic, no atomics).
#include "common.cuh"

#include <cstdlib>

namespace rlb {

constexpr int kNormWarps = 4;

template <typename T>
__global__ void __launch_bounds__(kNormWarps * 32)
rmsnorm_fwd_kernel(const T* __restrict__ x, const T* __restrict__ delta, const T* __restrict__ w,
                   T* __restrict__ y, T* __restrict__ s_out, float* __restrict__ rstd, int rows, int H,
                   float eps) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  pdl_launch_dependents();
  if (row >= rows) return;
  const T* xr = x + (size_t)row * H;
  const T* dr = delta ? delta + (size_t)row * H : nullptr;
  T* sr = s_out ? s_out + (size_t)row * H : nullptr;
  float ss = 0.f;
  const bool vec = (sizeof(T) == 2) && (H % 8 == 0);
  if (vec) {
    const int nv = H / 8;
    for (int j = lane; j < nv; j += 32) {
      float f[8];
      unpack8(reinterpret_cast<const bf16x8*>(xr)[j], f);
      if (dr) {
        float g[8];
        unpack8(reinterpret_cast<const bf16x8*>(dr)[j], g);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] += g[i];
        bf16x8 p = pack8(f);
        reinterpret_cast<bf16x8*>(sr)[j] = p;
        unpack8(p, f);  // normalise the rounded sum that is stored
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
  } else {
    for (int j = lane; j < H; j += 32) {
      float v = to_f(xr[j]);
      if (dr) {
        T s = from_f<T>(v + to_f(dr[j]));
        sr[j] = s;
        v = to_f(s);
      }
      ss += v * v;
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / H + eps);
  if (lane == 0) rstd[row] = r;
  const T* src = dr ? sr : xr;
  __syncwarp();
  T* yr = y + (size_t)row * H;
  if (vec) {
    const int nv = H / 8;
    for (int j = lane; j < nv; j += 32) {
      float f[8], g[8];
      unpack8(reinterpret_cast<const bf16x8*>(src)[j], f);
      unpack8(reinterpret_cast<const bf16x8*>(w)[j], g);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = f[i] * r * g[i];
      reinterpret_cast<bf16x8*>(yr)[j] = pack8(f);
    }
  } else {
    for (int j = lane; j < H; j += 32) yr[j] = from_f<T>(to_f(src[j]) * r * to_f(w[j]));
  }
}

// Few-row variant (decode batches): one 128-thread CTA per row so that a batch of
// tens of rows still spreads over many SMs.  bf16 rows with H % 8 == 0 only.
__global__ void __launch_bounds__(128)
rmsnorm_fwd_rowcta_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ delta,
                          const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                          __nv_bfloat16* __restrict__ s_out, float* __restrict__ rstd, int H, float eps) {
  pdl_launch_dependents();
  __shared__ float red[32];
  const int row = blockIdx.x;
  const int nv = H / 8;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + (size_t)row * H);
  const bf16x8* dr = delta ? reinterpret_cast<const bf16x8*>(delta + (size_t)row * H) : nullptr;
  bf16x8* sr = s_out ? reinterpret_cast<bf16x8*>(s_out + (size_t)row * H) : nullptr;
  constexpr int kMaxV = 8;  // vectors per thread kept in registers (H <= 8192)
  float v[kMaxV][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxV; ++k) {
    const int j = threadIdx.x + k * 128;
    if (j < nv) {
      unpack8(xr[j], v[k]);
      if (dr) {
        float d[8];
        unpack8(dr[j], d);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[k][i] += d[i];
        bf16x8 p = pack8(v[k]);
        sr[j] = p;
        unpack8(p, v[k]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[k][i] * v[k][i];
    }
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + (size_t)row * H);
  const bf16x8* wv = reinterpret_cast<const bf16x8*>(w);
#pragma unroll
  for (int k = 0; k < kMaxV; ++k) {
    const int j = threadIdx.x + k * 128;
    if (j < nv) {
      float g[8];
      unpack8(wv[j], g);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[k][i] = v[k][i] * r * g[i];
      yr[j] = pack8(v[k]);
    }
  }
}

// dx = r * dy * w - x * r^3 * sum(dy * w * x) / H   (+ ds)
// dw_partial[cta][h] = sum over this CTA's rows of dy * x * r
template <typename T>
__global__ void __launch_bounds__(kNormWarps * 32)
rmsnorm_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w,
                   const float* __restrict__ rstd, const T* __restrict__ ds, T* __restrict__ dx,
                   float* __restrict__ dw_partial, int rows, int H) {
  extern __shared__ float acc[];  // [kNormWarps][H]
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* my = acc + (size_t)wid * H;
  for (int j = lane; j < H; j += 32) my[j] = 0.f;
  __syncwarp();
  const bool vec = (sizeof(T) == 2) && (H % 8 == 0);
  for (int row = blockIdx.x * kNormWarps + wid; row < rows; row += gridDim.x * kNormWarps) {
    const T* dyr = dy + (size_t)row * H;
    const T* xr = x + (size_t)row * H;
    const float r = rstd[row];
    float dot = 0.f;
    if (vec) {
      for (int j = lane; j < H / 8; j += 32) {
        float a[8], b[8], c[8];
        unpack8(reinterpret_cast<const bf16x8*>(dyr)[j], a);
        unpack8(reinterpret_cast<const bf16x8*>(xr)[j], b);
        unpack8(reinterpret_cast<const bf16x8*>(w)[j], c);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot += a[i] * c[i] * b[i];
      }
    } else {
      for (int j = lane; j < H; j += 32) dot += to_f(dyr[j]) * to_f(w[j]) * to_f(xr[j]);
    }
    dot = warp_sum(dot);
    const float c3 = dot * r * r * r / H;
    T* dxr = dx + (size_t)row * H;
    const T* dsr = ds ? ds + (size_t)row * H : nullptr;
    if (vec) {
      for (int j = lane; j < H / 8; j += 32) {
        float a[8], b[8], c[8], o[8];
        unpack8(reinterpret_cast<const bf16x8*>(dyr)[j], a);
        unpack8(reinterpret_cast<const bf16x8*>(xr)[j], b);
        unpack8(reinterpret_cast<const bf16x8*>(w)[j], c);
        float e[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (dsr) unpack8(reinterpret_cast<const bf16x8*>(dsr)[j], e);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          o[i] = r * a[i] * c[i] - b[i] * c3 + e[i];
          my[j * 8 + i] += a[i] * b[i] * r;
        }
        reinterpret_cast<bf16x8*>(dxr)[j] = pack8(o);
      }
    } else {
      for (int j = lane; j < H; j += 32) {
        float a = to_f(dyr[j]), b = to_f(xr[j]);
        float o = r * a * to_f(w[j]) - b * c3 + (dsr ? to_f(dsr[j]) : 0.f);
        dxr[j] = from_f<T>(o);
        my[j] += a * b * r;
      }
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < H; j += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kNormWarps; ++k) s += acc[(size_t)k * H + j];
    dw_partial[(size_t)blockIdx.x * H + j] = s;
  }
}

__global__ void reduce_rows_kernel(const float* __restrict__ part, float* __restrict__ out, int n_rows, int H) {
  int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= H) return;
  float s = 0.f;
  for (int i = 0; i < n_rows; ++i) s += part[(size_t)i * H + j];
  out[j] = s;
}

}  // namespace rlb

using namespace rlb;

// Few-row (decode) batches take the one-CTA-per-row kernel unless RLB_NORM_ROWCTA=0.
static bool use_rowcta(const at::Tensor& x, int H, int rows) {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("RLB_NORM_ROWCTA");
    on = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return on == 1 && x.scalar_type() == at::kBFloat16 && H % 8 == 0 && H <= 8192 && rows < 4 * num_sms();
}

static void check_rows(const at::Tensor& x, const at::Tensor& w) {
  RLB_CHECK(x.is_cuda() && x.dim() == 2 && x.is_contiguous(), "norm input must be a contiguous 2-D CUDA tensor");
  RLB_CHECK(w.dim() == 1 && w.size(0) == x.size(1) && w.scalar_type() == x.scalar_type(), "norm weight mismatch");
}

std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps) {
  check_rows(x, w);
  const c10::cuda::CUDAGuard g(x.device());
  const int rows = x.size(0), H = x.size(1);
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, rstd};
  if (use_rowcta(x, H, rows)) {
    rmsnorm_fwd_rowcta_kernel<<<rows, 128, 0, stream()>>>(
        (const __nv_bfloat16*)x.data_ptr(), nullptr, (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(),
        nullptr, rstd.data_ptr<float>(), H, (float)eps);
    RLB_CUDA_CHECK(cudaGetLastError());
    return {y, rstd};
  }
  dim3 grid((rows + kNormWarps - 1) / kNormWarps);
  RLB_DISPATCH_FLOAT(x.scalar_type(), "rmsnorm_fwd", [&] {
    rmsnorm_fwd_kernel<scalar_t><<<grid, kNormWarps * 32, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), nullptr, (const scalar_t*)w.data_ptr(), (scalar_t*)y.data_ptr(), nullptr,
        rstd.data_ptr<float>(), rows, H, (float)eps);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {y, rstd};
}

std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, at::Tensor delta, at::Tensor w, double eps) {
  check_rows(x, w);
  RLB_CHECK(delta.sizes() == x.sizes() && delta.is_contiguous(), "delta shape mismatch");
  const c10::cuda::CUDAGuard g(x.device());
  const int rows = x.size(0), H = x.size(1);
  auto y = at::empty_like(x);
  auto s = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  if (rows == 0) return {y, s, rstd};
  if (use_rowcta(x, H, rows)) {
    rmsnorm_fwd_rowcta_kernel<<<rows, 128, 0, stream()>>>(
        (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)delta.data_ptr(), (const __nv_bfloat16*)w.data_ptr(),
        (__nv_bfloat16*)y.data_ptr(), (__nv_bfloat16*)s.data_ptr(), rstd.data_ptr<float>(), H, (float)eps);
    RLB_CUDA_CHECK(cudaGetLastError());
    return {y, s, rstd};
  }
  dim3 grid((rows + kNormWarps - 1) / kNormWarps);
  RLB_DISPATCH_FLOAT(x.scalar_type(), "add_rmsnorm_fwd", [&] {
    rmsnorm_fwd_kernel<scalar_t><<<grid, kNormWarps * 32, 0, stream()>>>(
        (const scalar_t*)x.data_ptr(), (const scalar_t*)delta.data_ptr(), (const scalar_t*)w.data_ptr(),
        (scalar_t*)y.data_ptr(), (scalar_t*)s.data_ptr(), rstd.data_ptr<float>(), rows, H, (float)eps);
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {y, s, rstd};
}

static std::vector<at::Tensor> rmsnorm_bwd_impl(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                                                c10::optional<at::Tensor> ds) {
  check_rows(x, w);
  RLB_CHECK(dy.sizes() == x.sizes() && dy.is_contiguous(), "dy shape mismatch");
  const c10::cuda::CUDAGuard g(x.device());
  const int rows = x.size(0), H = x.size(1);
  auto dx = at::empty_like(x);
  auto dw = at::zeros({H}, x.options().dtype(at::kFloat));
  if (rows == 0) return {dx, dw};
  int ctas = std::min((rows + kNormWarps - 1) / kNormWarps, 2 * num_sms());
  size_t smem = (size_t)kNormWarps * H * sizeof(float);
  RLB_CHECK(smem <= 200 * 1024, "hidden size too large for rmsnorm_bwd shared accumulator");
  auto part = at::empty({ctas, H}, x.options().dtype(at::kFloat));
  const void* dsp = (ds.has_value() && ds->defined()) ? ds->data_ptr() : nullptr;
  RLB_DISPATCH_FLOAT(x.scalar_type(), "rmsnorm_bwd", [&] {
    auto kern = rmsnorm_bwd_kernel<scalar_t>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    kern<<<ctas, kNormWarps * 32, smem, stream()>>>(
        (const scalar_t*)dy.data_ptr(), (const scalar_t*)x.data_ptr(), (const scalar_t*)w.data_ptr(),
        rstd.data_ptr<float>(), (const scalar_t*)dsp, (scalar_t*)dx.data_ptr(), part.data_ptr<float>(), rows, H);
  });
  reduce_rows_kernel<<<(H + 255) / 256, 256, 0, stream()>>>(part.data_ptr<float>(), dw.data_ptr<float>(), ctas, H);
  RLB_CUDA_CHECK(cudaGetLastError());
  return {dx, dw};
}

std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd) {
  return rmsnorm_bwd_impl(dy, x, w, rstd, c10::nullopt);
}

std::vector<at::Tensor> rmsnorm_bwd_add(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                                        c10::optional<at::Tensor> ds) {
  return rmsnorm_bwd_impl(dy, x, w, rstd, ds);
}

// ---------------------------------------------------------------------------
// Allocation-free C entry point (declared in noalloc.h, where its contract is
// described; it has no counterpart in the reference).  It launches the same
// backward kernels as rmsnorm_bwd above, with the per-CTA dw partials placed in
// a static device array instead of a freshly allocated tensor.
#include <cstdio>
#include <mutex>

#include "noalloc.h"

namespace rlb {
static __device__ __align__(256) float g_noalloc_rmsnorm_partials[RLB_NOALLOC_MAX_CTAS * RLB_NOALLOC_MAX_HIDDEN];
}  // namespace rlb

namespace {
constexpr int kNoallocMaxDevices = 64;
float* g_noalloc_scratch[kNoallocMaxDevices] = {nullptr};
std::mutex g_noalloc_mu;
thread_local char g_noalloc_err[256] = "";

int noalloc_fail(int code, const char* msg) {
  std::snprintf(g_noalloc_err, sizeof(g_noalloc_err), "%s", msg);
  return code;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
}  // namespace

extern "C" __attribute__((visibility("default"))) const char* rlb_noalloc_last_error(void) { return g_noalloc_err; }

extern "C" __attribute__((visibility("default"))) int rlb_rmsnorm_bwd_noalloc(const void* dy, const void* x,
                                                                            const void* w, const float* rstd,
                                                                            void* dx, float* dw, int rows,
                                                                            int hidden, cudaStream_t stream) {
  if (!dy || !x || !w || !rstd || !dx || !dw) return noalloc_fail(1, "rlb_rmsnorm_bwd_noalloc: null pointer");
  if (rows < 0 || hidden <= 0) return noalloc_fail(1, "rlb_rmsnorm_bwd_noalloc: rows must be >= 0 and hidden > 0");
  if (hidden > RLB_NOALLOC_MAX_HIDDEN) {
    std::snprintf(g_noalloc_err, sizeof(g_noalloc_err),
                  "rlb_rmsnorm_bwd_noalloc: hidden=%d exceeds the static scratch maximum of %d", hidden,
                  RLB_NOALLOC_MAX_HIDDEN);
    return 2;
  }
  if (hidden % 8 == 0 && !(aligned(dy, 16) && aligned(x, 16) && aligned(w, 16) && aligned(dx, 16)))
    return noalloc_fail(3, "rlb_rmsnorm_bwd_noalloc: dy, x, w and dx must be 16-byte aligned");
  if (!aligned(rstd, 4) || !aligned(dw, 4)) return noalloc_fail(3, "rlb_rmsnorm_bwd_noalloc: rstd/dw misaligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(4, cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoallocMaxDevices) return noalloc_fail(4, "rlb_rmsnorm_bwd_noalloc: device index too large");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_scratch[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, rlb::g_noalloc_rmsnorm_partials);
      if (e != cudaSuccess || p == nullptr) return noalloc_fail(5, cudaGetErrorString(e));
      g_noalloc_scratch[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_scratch[dev];
  }
  if (rows == 0) {
    e = cudaMemsetAsync(dw, 0, sizeof(float) * hidden, stream);
    return e == cudaSuccess ? 0 : noalloc_fail(6, cudaGetErrorString(e));
  }
  const int ctas = std::min((rows + kNormWarps - 1) / kNormWarps, RLB_NOALLOC_MAX_CTAS);
  const size_t smem = (size_t)kNormWarps * hidden * sizeof(float);
  auto kern = rmsnorm_bwd_kernel<__nv_bfloat16>;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return noalloc_fail(6, cudaGetErrorString(e));
  }
  kern<<<ctas, kNormWarps * 32, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
      static_cast<const __nv_bfloat16*>(w), rstd, nullptr, static_cast<__nv_bfloat16*>(dx), scratch, rows, hidden);
  reduce_rows_kernel<<<(hidden + 255) / 256, 256, 0, stream>>>(scratch, dw, ctas, hidden);
  e = cudaGetLastError();
  if (e != cudaSuccess) return noalloc_fail(6, cudaGetErrorString(e));
  return 0;
}
