// Tensor-parallel decode: all-reduce of the row-parallel projection's partial
// sums fused with the residual add and the next RMSNorm, over NVLink peer
// memory (replaces NCCL all-reduce + add_rms_norm after every o_proj / down_proj
// of a decode step).
//
// One CTA per token row b:
//   1. copy this rank's partial row into its symmetric slot (parity of the call)
//      and publish (release, system scope) the call's epoch in every rank's
//      flag word for (this rank, row b);
//   2. wait (bounded) until every rank has published row b;
//   3. sum the n partial rows in rank order (identical bits on every rank),
//      add the residual, write the new residual and RMSNorm(new residual) * w.
// The epoch comes from a device counter (read at kernel start, advanced by the
// last CTA to finish), so the kernel replays inside CUDA graphs.  Slots are
// double-buffered by epoch parity: a rank rewrites a slot row two calls later,
// after it saw every peer publish that row for the call in between, which each
// peer does only after it finished reading the slot.  On a wait timeout an
// error word is set (decode_ar_error_flag) and the row is reduced with what is there.
#include "common.cuh"

namespace rlb {
namespace dar {

__device__ int g_dar_error = 0;
constexpr int kMax = 8;

struct Peers {
  __nv_bfloat16* slot[kMax];  // every rank's [2][cap][H] bf16 slots
  uint32_t* flag[kMax];       // every rank's [n][cap] u32 flag words (index src * cap + row)
  long long wait;             // bound of the wait on every peer's flag (cycles)
};

__global__ void __launch_bounds__(256)
ar_add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ partial, __nv_bfloat16* __restrict__ resid,
                      const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H, float eps,
                      Peers pe, int n, int me, int cap, uint32_t* __restrict__ ctr, unsigned int* __restrict__ done) {
  __shared__ float red[32];
  __shared__ uint32_t ep_s;
  __shared__ __nv_bfloat16* slot_s[kMax];
  __shared__ uint32_t* flag_s[kMax];
  const int b = blockIdx.x;
  if (threadIdx.x == 0) ep_s = *reinterpret_cast<volatile uint32_t*>(ctr) + 1u;
  if (threadIdx.x < kMax) {  // peer pointers in shared memory: indexed by rank without a local copy
#pragma unroll
    for (int r = 0; r < kMax; ++r)
      if (r == (int)threadIdx.x) {
        slot_s[r] = pe.slot[r];
        flag_s[r] = pe.flag[r];
      }
  }
  __syncthreads();
  const uint32_t ep = ep_s;
  const int par = ep & 1;
  const long long rowoff = ((long long)par * cap + b) * H;
  // 1. publish this rank's partial row
  const uint4* src = reinterpret_cast<const uint4*>(partial + (long long)b * H);
  uint4* mine = reinterpret_cast<uint4*>(slot_s[me] + rowoff);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) mine[c] = src[c];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < n) {
    uint32_t* f = flag_s[threadIdx.x] + (long long)me * cap + b;
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(f), "r"(ep) : "memory");
  }
  // 2. wait for every rank's row b
  if (threadIdx.x < n) {
    const uint32_t* f = flag_s[me] + (long long)threadIdx.x * cap + b;
    const long long t0 = clock64();
    for (;;) {
      uint32_t x;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(x) : "l"(f) : "memory");
      if ((int)(x - ep) >= 0) break;
      if (clock64() - t0 > pe.wait) {
        atomicExch(&g_dar_error, 1);
        break;
      }
    }
  }
  __syncthreads();
  // 3. reduce in rank order, residual add, RMSNorm
  float ss = 0.f;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < n; ++r) {
      float f[8];
      const uint4 v = reinterpret_cast<const uint4*>(slot_s[r] + rowoff)[c];
      unpack8(*reinterpret_cast<const bf16x8*>(&v), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
    // the reduced projection is rounded to bf16 as the library all-reduce would be
    float rs[8];
    const uint4 rv = reinterpret_cast<const uint4*>(resid + (long long)b * H)[c];
    unpack8(*reinterpret_cast<const bf16x8*>(&rv), rs);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = __bfloat162float(__float2bfloat16_rn(acc[e]));
      acc[e] = __bfloat162float(__float2bfloat16_rn(rs[e] + a));
      ss += acc[e] * acc[e];
    }
    *reinterpret_cast<bf16x8*>(resid + (long long)b * H + c * 8) = pack8(acc);
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float x[8], wv[8];
    const uint4 rv = reinterpret_cast<const uint4*>(resid + (long long)b * H)[c];
    const uint4 ww = reinterpret_cast<const uint4*>(w)[c];
    unpack8(*reinterpret_cast<const bf16x8*>(&rv), x);
    unpack8(*reinterpret_cast<const bf16x8*>(&ww), wv);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = x[e] * inv * wv[e];
    *reinterpret_cast<bf16x8*>(out + (long long)b * H + c * 8) = pack8(x);
  }
  // the last CTA advances the epoch counter (every CTA has read it by then)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(done, 1u);
    if (prev == gridDim.x - 1) {
      *done = 0u;
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(ctr) = ep;
    }
  }
}

}  // namespace dar
}  // namespace rlb

using namespace rlb;

// partial [B, H] bf16 (this rank's row-parallel output); resid [B, H] bf16 is
// updated in place; returns RMSNorm(resid + sum_r partial_r) * w.
at::Tensor ar_add_rmsnorm(at::Tensor partial, at::Tensor resid, at::Tensor w, double eps, std::vector<int64_t> slots,
                          std::vector<int64_t> flags, int64_t me, int64_t cap, at::Tensor ctr, at::Tensor done) {
  TORCH_CHECK(partial.is_cuda() && partial.scalar_type() == at::kBFloat16 && partial.is_contiguous() &&
                  resid.is_contiguous() && resid.sizes() == partial.sizes() && w.is_contiguous(),
              "ar_add_rmsnorm: bf16 contiguous [B, H] tensors");
  const int B = partial.size(0), H = partial.size(1);
  TORCH_CHECK(H % 8 == 0 && w.numel() == H && B <= cap, "ar_add_rmsnorm: H % 8 == 0, rows <= capacity");
  const size_t n = slots.size();
  TORCH_CHECK(n >= 1 && n <= (size_t)dar::kMax && flags.size() == n, "ar_add_rmsnorm: 1..8 ranks");
  dar::Peers pe{};
  pe.wait = peer_wait_cycles();
  for (size_t i = 0; i < n; ++i) {
    pe.slot[i] = reinterpret_cast<__nv_bfloat16*>((uintptr_t)slots[i]);
    pe.flag[i] = reinterpret_cast<uint32_t*>((uintptr_t)flags[i]);
  }
  const c10::cuda::CUDAGuard guard(partial.device());
  auto out = at::empty_like(partial);
  if (B == 0) return out;
  dar::ar_add_rmsnorm_kernel<<<B, 256, 0, stream()>>>(
      (const __nv_bfloat16*)partial.data_ptr(), (__nv_bfloat16*)resid.data_ptr(), (const __nv_bfloat16*)w.data_ptr(),
      (__nv_bfloat16*)out.data_ptr(), H, (float)eps, pe, (int)n, (int)me, (int)cap,
      reinterpret_cast<uint32_t*>(ctr.data_ptr<int>()), reinterpret_cast<unsigned int*>(done.data_ptr<int>()));
  RLB_CUDA_CHECK(cudaGetLastError());
  return out;
}

int64_t decode_ar_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, dar::g_dar_error, sizeof(int)));
  if (reset) {
    const int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(dar::g_dar_error, &z, sizeof(int)));
  }
  return v;
}
