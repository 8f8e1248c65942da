// Shared device helpers for the rl_b200 sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#define RLB_CHECK(cond, msg) TORCH_CHECK((cond), "rl_b200: ", msg)
#define RLB_CUDA_CHECK(expr)                                                      \
  do {                                                                            \
    cudaError_t _e = (expr);                                                      \
    TORCH_CHECK(_e == cudaSuccess, "rl_b200 CUDA error: ", cudaGetErrorString(_e), \
                " at " __FILE__ ":", __LINE__);                                   \
  } while (0)

namespace rlb {

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Upper bound, in SM clock cycles, of every wait on a flag written by ANOTHER rank
// or by a copy engine (fused collectives, expert dispatch, context-parallel K/V
// arrival).  Kernels receive it as an argument; on expiry they set their error
// word and return instead of spinning.  Default 4e9 cycles (about 2 s at 2 GHz);
// tests lower it to make a wait run out quickly.  Defined in bindings.cpp.
int64_t peer_wait_cycles();
void set_peer_wait_cycles(int64_t cycles);

// Bounds checks of data-dependent indices (row ids, cache slots, block-table
// entries, expert rows) for the bounds-checked debug build (-DRLB_DEBUG_BOUNDS,
// built as rl_b200._C_debug).  RLB_IN_BOUNDS(i, n, site) is true when
// 0 <= i < n; in the debug build a false result records (site << 40 | low 40 bits
// of i) in this translation unit's error word (the first failure wins) and the
// caller skips the access, so an index bug is reported instead of touching
// memory outside the tensor.  In the release build it is the constant true.
// site codes (the error word's top bits)
constexpr int kBoundsKvSlot = 1;       // KV-cache slot of a written token
constexpr int kBoundsBlockTable = 2;   // paged-attention block-table entry
constexpr int kBoundsEpRow = 3;        // expert-parallel destination row / rank / source row
constexpr int kBoundsRouterRow = 4;    // MoE router expert-grouped row
#ifdef RLB_DEBUG_BOUNDS
static __device__ unsigned long long g_rlb_bounds_err = 0ull;
__device__ __forceinline__ bool rlb_in_bounds(long long i, long long n, int site) {
  if (i >= 0 && i < n) return true;
  atomicCAS(&g_rlb_bounds_err, 0ull,
            ((unsigned long long)site << 40) | ((unsigned long long)i & ((1ull << 40) - 1ull)));
  return false;
}
#define RLB_IN_BOUNDS(i, n, site) rlb_in_bounds((long long)(i), (long long)(n), (site))
// host side: read (and optionally clear) this translation unit's error word
static inline int64_t rlb_bounds_error(bool reset) {
  unsigned long long v = 0;
  cudaMemcpyFromSymbol(&v, g_rlb_bounds_err, sizeof(v));
  if (reset && v) {
    const unsigned long long z = 0;
    cudaMemcpyToSymbol(g_rlb_bounds_err, &z, sizeof(z));
  }
  return (int64_t)v;
}
#else
#define RLB_IN_BOUNDS(i, n, site) true
static inline int64_t rlb_bounds_error(bool) { return 0; }
#endif

inline int num_sms() {
  static int n = -1;
  if (n < 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Programmatic dependent launch.  A kernel that calls pdl_launch_dependents()
// lets the kernel launched after it on the same stream WITH programmatic stream
// serialization (the decode-shaped GEMM) start early: that kernel runs its
// independent prologue (barrier set-up, tensor-memory allocation, the weight
// stream) and calls pdl_wait() before it reads anything this kernel wrote;
// pdl_wait() returns once every earlier kernel completed and its writes are
// visible.  For a kernel launched without the attribute both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `red` must hold >= 32 floats.  All threads get the result.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? red[lane] : 0.f;
  r = warp_sum(r);
  return r;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = (lane < nw) ? red[lane] : -INFINITY;
  r = warp_max(r);
  return r;
}

// 8 x bf16 packed in 16 bytes
struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ void unpack8(const bf16x8& p, float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p.v[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ bf16x8 pack8(const float* f) {
  bf16x8 p;
#pragma unroll
  for (int i = 0; i < 4; ++i) p.v[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return p;
}

// Element load / store helpers generic over float / bf16 / half
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Counter-based 32-bit hash ("lowbias32", C. Wellons, 2018) used for sampling noise.
__device__ __forceinline__ uint32_t hash32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// Uniform in (0, 1) from (seed, stream, counter): never exactly 0 or 1.
__device__ __forceinline__ float uniform01(uint32_t seed, uint32_t stream, uint32_t counter) {
  uint32_t h = hash32(seed ^ hash32(stream * 0x9E3779B9u ^ hash32(counter + 0x85EBCA6Bu)));
  return (static_cast<float>(h >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

}  // namespace rlb

#define RLB_DISPATCH_FLOAT(TYPE, NAME, ...)                                 \
  [&] {                                                                     \
    if ((TYPE) == at::kBFloat16) {                                          \
      using scalar_t = __nv_bfloat16;                                       \
      return __VA_ARGS__();                                                 \
    } else if ((TYPE) == at::kHalf) {                                       \
      using scalar_t = __half;                                              \
      return __VA_ARGS__();                                                 \
    } else if ((TYPE) == at::kFloat) {                                      \
      using scalar_t = float;                                               \
      return __VA_ARGS__();                                                 \
    } else {                                                                \
      TORCH_CHECK(false, NAME, ": unsupported dtype ", (TYPE));             \
    }                                                                       \
  }()
