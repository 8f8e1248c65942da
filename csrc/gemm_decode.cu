// Decode-shaped GEMM on the 5th-generation tensor cores (sm_100a):
//
//   out[Mb, N] (bf16) = x[Mb, K] (bf16) x W[N, K]^T (bf16),   Mb <= 256
//
// A rollout decode step multiplies a few dozen to a few hundred token rows by
// every weight matrix of the model, so the product is bound by streaming W
// from HBM.  Library GEMMs tile the few rows poorly (1.9 - 2.8 TB/s on the
// 8B attention projections); this kernel computes the TRANSPOSED product so
// that W supplies the 128-row MMA operand:
//
//   D^T[128-row tile of W, BN] = W tile (A, K-major) x x (B, K-major),
//
// with BN = Mb rounded up to 32/64/128/256 (TMA fills the missing x rows with
// zeros).  The K dimension is split into S ranges so that (N/128) x S work items
// fill every SM; warp 0 streams W and x tiles with TMA (no multicast) through
// a deep shared-memory ring, warp 1 issues tcgen05.mma into double-buffered
// TMEM accumulators, warps 2-5 drain them.  With S > 1 every split stores its
// fp32 partial tile to a workspace slice and bumps a per-tile arrival counter;
// the last split to arrive sums the S slices in split order (deterministic),
// writes bf16 rows and resets the counter.  All waits are bounded; the
// counters are shared by every call on a device, so calls must not overlap on
// the GPU (one stream).
#include "tc_common.cuh"

#include <mutex>
#include <unordered_map>

namespace rlb {
namespace dec {

__device__ int g_dec_error = 0;

using namespace rlb::tc;

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                   __nv_bfloat16* __restrict__ out, float* __restrict__ ws, int* __restrict__ counters, int Mb, int N,
                   int K, int S, int kb_per) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16(BM, BN);
  extern __shared__ uint8_t smem_raw[];
  __shared__ int last_flag;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + STAGES * (A_BYTES + B_BYTES));
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;
  const uint32_t bar_tempty = bar_tfull + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (N + BM - 1) / BM;
  const int num_kb = (K + BK - 1) / BK;
  const int items = num_m * S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int item = blockIdx.x; item < items && !*abort_flag; item += gridDim.x) {
        const int mt = item % num_m, split = item / num_m;
        const int kb0 = split * kb_per, nkb = min(num_kb, kb0 + kb_per) - kb0;
        // every CTA reads the same x tiles: start each CTA at a different K-block so
        // the ~148 concurrent readers of one x tile (an L2 hot spot) spread out
        const int rot = nkb > 0 ? (int)(blockIdx.x % nkb) : 0;
        for (int kk = 0; kk < nkb; ++kk, ++it) {
          const int kb = kb0 + (kk + rot) % nkb;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_err(bar_empty + 8 * s, ph ^ 1, abort_flag, &g_dec_error, 1)) break;
          mbar_expect_tx(bar_full + 8 * s, A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmap_w, bar_full + 8 * s, kb * BK, mt * BM);
          tma_load_2d(sB + s * B_BYTES, &tmap_x, bar_full + 8 * s, kb * BK, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      for (int item = blockIdx.x; item < items && !*abort_flag; item += gridDim.x, ++local) {
        const int split = item / num_m;
        const int kb0 = split * kb_per, nkb = min(num_kb, kb0 + kb_per) - kb0;
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait_err(bar_tempty + 8 * acc, aph ^ 1, abort_flag, &g_dec_error, 1)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        bool ok = true;
        for (int kk = 0; kk < nkb; ++kk, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_err(bar_full + 8 * s, ph, abort_flag, &g_dec_error, 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + s * A_BYTES, b0 = sB + s * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(tmem_d, desc_kmajor_sw128(a0 + k * 32), desc_kmajor_sw128(b0 + k * 32), IDESC,
                      (kk > 0 || k > 0) ? 1u : 0u);
          umma_commit(bar_empty + 8 * s);
        }
        if (!ok) break;
        umma_commit(bar_tfull + 8 * acc);
      }
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    int local = 0;
    for (int item = blockIdx.x; item < items; item += gridDim.x, ++local) {
      const int mt = item % num_m, split = item / num_m;
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait_err(bar_tfull + 8 * acc, aph, abort_flag, &g_dec_error, 1)) break;
      tc_fence_after();
      const int n = mt * BM + quad * 32 + lane;  // weight row = output column
      const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      if (S == 1) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + c * 32, r);
          if (n < N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int b = c * 32 + j;
              if (b < Mb) out[(long long)b * N + n] = __float2bfloat16_rn(__uint_as_float(r[j]));
            }
          }
        }
        tc_fence_before();
      } else {
        float* slice = ws + (long long)split * Mb * N;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + c * 32, r);
          if (n < N) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int b = c * 32 + j;
              if (b < Mb) __stcg(slice + (long long)b * N + n, __uint_as_float(r[j]));
            }
          }
        }
        tc_fence_before();
        __threadfence();
        asm volatile("bar.sync 1, 128;\n" ::: "memory");
        if (warp == 2 && lane == 0) last_flag = (atomicAdd(counters + mt, 1) == S - 1) ? 1 : 0;
        asm volatile("bar.sync 1, 128;\n" ::: "memory");
        if (last_flag) {
          __threadfence();
          if (n < N) {
            // 8 batch rows at a time: 8 independent L2 loads in flight per split
#pragma unroll 1
            for (int b0 = 0; b0 < Mb; b0 += 8) {
              float acc[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) acc[q] = 0.f;
#pragma unroll 1
              for (int sp = 0; sp < S; ++sp) {
                float t[8];
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  t[q] = (b0 + q < Mb) ? __ldcg(ws + ((long long)sp * Mb + b0 + q) * N + n) : 0.f;
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[q] += t[q];
              }
#pragma unroll
              for (int q = 0; q < 8; ++q)
                if (b0 + q < Mb) out[(long long)(b0 + q) * N + n] = __float2bfloat16_rn(acc[q]);
            }
          }
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
          if (warp == 2 && lane == 0) counters[mt] = 0;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

}  // namespace dec
}  // namespace rlb

using namespace rlb;

namespace {
struct DecodeScratch {
  at::Tensor ws, counters;
};
std::mutex g_scratch_mu;
std::unordered_map<int, DecodeScratch> g_scratch;

DecodeScratch& scratch_for(const at::Tensor& like, long long ws_elems, int counters) {
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  auto& sc = g_scratch[like.get_device()];
  if (!sc.ws.defined() || sc.ws.numel() < ws_elems)
    sc.ws = at::empty({std::max<long long>(ws_elems, 1 << 20)}, like.options().dtype(at::kFloat));
  if (!sc.counters.defined() || sc.counters.numel() < counters)
    sc.counters = at::zeros({std::max(counters, 4096)}, like.options().dtype(at::kInt));
  return sc;
}

template <int BN, int STAGES>
void launch_decode(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int Mb, int N, int K) {
  const int num_m = (N + tc::BM - 1) / tc::BM;
  const int num_kb = (K + tc::BK - 1) / tc::BK;
  const int sms = num_sms();
  // split K so that the work items fill the SMs in near-whole waves, each item
  // streaming at least 4 K-blocks of W
  int S = 1;
  double best = 0.0;
  for (int s = 1; s <= std::min(16, std::max(1, num_kb / 4)); ++s) {
    const int items = num_m * s;
    const double eff = (double)items / ((double)((items + sms - 1) / sms) * sms);
    if (eff > best + 0.03) {
      best = eff;
      S = s;
    }
  }
  const int kb_per = (num_kb + S - 1) / S;
  S = (num_kb + kb_per - 1) / kb_per;
  float* ws = nullptr;
  int* counters = nullptr;
  if (S > 1) {
    auto& sc = scratch_for(x, (long long)S * Mb * N, num_m);
    ws = sc.ws.data_ptr<float>();
    counters = sc.counters.data_ptr<int>();
  }
  const CUtensorMap tw = make_tmap_2d(w.data_ptr(), N, K, tc::BM);
  const CUtensorMap tx = make_tmap_2d(x.data_ptr(), Mb, K, BN);
  const int smem = STAGES * (tc::BM * tc::BK * 2 + BN * tc::BK * 2) + 1024 + 256;
  auto kern = dec::gemm_decode_kernel<BN, STAGES>;
  RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int grid = std::min(num_m * S, sms);
  kern<<<grid, 192, smem, stream()>>>(tw, tx, (__nv_bfloat16*)out.data_ptr(), ws, counters, Mb, N, K, S, kb_per);
  RLB_CUDA_CHECK(cudaGetLastError());
}
}  // namespace

at::Tensor gemm_decode(at::Tensor x, at::Tensor w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "rl_b200 gemm_decode: bf16 CUDA operands expected");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "rl_b200 gemm_decode: x [Mb,K], w [N,K]");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous(), "rl_b200 gemm_decode: operands must be contiguous");
  const int Mb = x.size(0), N = w.size(0), K = x.size(1);
  TORCH_CHECK(Mb >= 1 && Mb <= 256, "rl_b200 gemm_decode: 1..256 rows");
  TORCH_CHECK(K % 8 == 0 && K > 0, "rl_b200 gemm_decode: K must be a positive multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "rl_b200 gemm_decode: operands must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty({Mb, N}, x.options());
  if (N == 0) return out;
  if (Mb <= 32) launch_decode<32, 10>(x, w, out, Mb, N, K);
  else if (Mb <= 64) launch_decode<64, 8>(x, w, out, Mb, N, K);
  else if (Mb <= 128) launch_decode<128, 6>(x, w, out, Mb, N, K);
  else launch_decode<256, 4>(x, w, out, Mb, N, K);
  return out;
}

int64_t gemm_decode_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, dec::g_dec_error, sizeof(int)));
  if (reset) {
    const int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(dec::g_dec_error, &z, sizeof(int)));
  }
  return v;
}
