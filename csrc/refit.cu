// Train -> rollout weight refit: reshard from the training tensor-parallel
// layout into the generation layout by loading the training shards straight
// out of the peer GPUs' HBM (CUDA IPC mappings of their flat parameter
// buffers, NVLink / NVSwitch), fused with either the bf16 copy or the 128x128
// block-scaled e4m3 quantisation of the destination weights.
//
// The host turns the layout change into a list of 2-D tasks (see
// rl_b200/weight_sync/reshard.py); every task is
//   { src_addr, src_ld, dst_off, dst_ld, rows, cols, scale_off, 0 }
// where src_addr is the device address (bytes; the IPC mapping for a peer
// shard) of the region's first bf16 element and the rest count ELEMENTS.  A copy task moves
// rows x cols bf16 elements with 16-byte vectors (offsets, leading dims and
// cols are multiples of 8 elements); a quant task is one <=128 x <=128 block of
// a destination weight: block amax -> scale = amax / 448 (optionally rounded up
// to a power of two) -> e4m3 values at dst_off, fp32 scale at scale_off.
//
// Reference counterpart: the NCCL broadcast / send-recv reshard
// (nemo_rl/weight_sync/xferdtensor_python.py:642-668) followed by the torch
// blockwise cast (nemo_rl/models/generation/vllm/quantization/fp8.py:756).
#include "common.cuh"

#include <cuda_fp8.h>

namespace rlb {
namespace refit {

struct Task {
  long long src_addr, src_ld, dst_off, dst_ld, rows, cols, scale_off, pad;
};

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr float kFp8Max = 448.f;

__device__ __forceinline__ uint4 ld_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// grid-stride over tasks; each CTA moves one task with 16-byte vectors,
// kUnroll loads in flight per thread (peer loads have microseconds of latency)
__global__ void __launch_bounds__(kThreads)
copy_kernel(const Task* __restrict__ tasks, long long ntasks, __nv_bfloat16* __restrict__ dst) {
  for (long long t = blockIdx.x; t < ntasks; t += gridDim.x) {
    const Task tk = tasks[t];
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(tk.src_addr);
    const long long vpr = tk.cols >> 3;  // 8-element vectors per row
    const long long nv = vpr * tk.rows;
    for (long long base = threadIdx.x; base < nv; base += (long long)kThreads * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const long long i = base + (long long)u * kThreads;
        if (i < nv) {
          const long long r = i / vpr, c = (i - r * vpr) << 3;
          v[u] = ld_v4(src + r * tk.src_ld + c);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const long long i = base + (long long)u * kThreads;
        if (i < nv) {
          const long long r = i / vpr, c = (i - r * vpr) << 3;
          *reinterpret_cast<uint4*>(dst + tk.dst_off + r * tk.dst_ld + c) = v[u];
        }
      }
    }
  }
}

__device__ __forceinline__ float pow2_ceil(float s) {
  uint32_t b = __float_as_uint(s);
  if (b & 0x007fffffu) b = (b & 0xff800000u) + 0x00800000u;
  return __uint_as_float(b & 0xff800000u);
}

// one <=128x128 block per task: 2048 8-element vectors, 8 per thread, held in
// registers between the amax reduction and the quantised store
__global__ void __launch_bounds__(kThreads)
quant_kernel(const Task* __restrict__ tasks, long long ntasks, uint8_t* __restrict__ q,
             float* __restrict__ scales, int pow2) {
  __shared__ float red[32];
  constexpr int kPer = 128 * 16 / kThreads;  // vectors per thread (8)
  for (long long t = blockIdx.x; t < ntasks; t += gridDim.x) {
    const Task tk = tasks[t];
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(tk.src_addr);
    const int vpr = (int)(tk.cols >> 3);
    const int nv = vpr * (int)tk.rows;
    uint4 v[kPer];
    float amax = 0.f;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = threadIdx.x + u * kThreads;
      v[u] = make_uint4(0, 0, 0, 0);
      if (i < nv) {
        const int r = i / vpr, c = (i - r * vpr) << 3;
        v[u] = ld_v4(src + (long long)r * tk.src_ld + c);
        float f[8];
        unpack8(*reinterpret_cast<const bf16x8*>(&v[u]), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
      }
    }
    amax = block_max(amax, red);
    float s = fmaxf(amax, 1e-12f) / kFp8Max;
    if (pow2) s = pow2_ceil(s);
    if (threadIdx.x == 0) scales[tk.scale_off] = s;
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = threadIdx.x + u * kThreads;
      if (i < nv) {
        const int r = i / vpr, c = (i - r * vpr) << 3;
        float f[8];
        unpack8(*reinterpret_cast<const bf16x8*>(&v[u]), f);
        uint32_t w[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t packed = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            // IEEE division (not a reciprocal multiply): the same e4m3 bytes as
            // the torch reference quantisation x / s
            const float x = fminf(fmaxf(__fdiv_rn(f[h * 4 + e], s), -kFp8Max), kFp8Max);
            const __nv_fp8_e4m3 b(x);
            packed |= (uint32_t)(*reinterpret_cast<const uint8_t*>(&b)) << (8 * e);
          }
          w[h] = packed;
        }
        *reinterpret_cast<uint2*>(q + tk.dst_off + (long long)r * tk.dst_ld + c) = make_uint2(w[0], w[1]);
      }
    }
    __syncthreads();  // red[] is reused by the next task's reduction
  }
}

}  // namespace refit
}  // namespace rlb

using namespace rlb;

namespace {
int grid_for(long long ntasks) {
  const long long cap = (long long)num_sms() * 4;
  return (int)std::max<long long>(1, std::min<long long>(ntasks, cap));
}
}  // namespace

// tasks: int64 [n, 8] on the device (source addresses already resolved to the
// training ranks' flat parameter buffers, own one included, 16-byte aligned
// rows); dst: bf16 flat buffer of the generation model.
void refit_copy(at::Tensor tasks, at::Tensor dst) {
  TORCH_CHECK(tasks.is_cuda() && tasks.scalar_type() == at::kLong && tasks.dim() == 2 && tasks.size(1) == 8,
              "refit_copy: tasks int64 [n, 8] on the device");
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == at::kBFloat16 && dst.is_contiguous(), "refit_copy: bf16 dst");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0, "refit_copy: dst must be 16-byte aligned");
  const long long n = tasks.size(0);
  if (n == 0) return;
  refit::copy_kernel<<<grid_for(n), refit::kThreads, 0, stream()>>>(
      reinterpret_cast<const refit::Task*>(tasks.data_ptr<int64_t>()), n,
      reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
  RLB_CUDA_CHECK(cudaGetLastError());
}

// q: uint8 (e4m3 bytes) flat buffer of the generation weights; scales: fp32.
void refit_quant_fp8(at::Tensor tasks, at::Tensor q, at::Tensor scales, bool pow2) {
  TORCH_CHECK(tasks.is_cuda() && tasks.scalar_type() == at::kLong && tasks.dim() == 2 && tasks.size(1) == 8,
              "refit_quant_fp8: tasks int64 [n, 8] on the device");
  TORCH_CHECK(q.is_cuda() && (q.scalar_type() == at::kByte || q.scalar_type() == at::kFloat8_e4m3fn),
              "refit_quant_fp8: q must be uint8 / e4m3");
  TORCH_CHECK(scales.is_cuda() && scales.scalar_type() == at::kFloat, "refit_quant_fp8: fp32 scales");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0, "refit_quant_fp8: q must be 16-byte aligned");
  const long long n = tasks.size(0);
  if (n == 0) return;
  refit::quant_kernel<<<grid_for(n), refit::kThreads, 0, stream()>>>(
      reinterpret_cast<const refit::Task*>(tasks.data_ptr<int64_t>()), n,
      reinterpret_cast<uint8_t*>(q.data_ptr()), scales.data_ptr<float>(), pow2 ? 1 : 0);
  RLB_CUDA_CHECK(cudaGetLastError());
}
