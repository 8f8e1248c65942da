// Decode-shaped GEMM on the 5th-generation tensor cores (sm_100a):
//
//   out[Mb, N] (bf16) = x[Mb, K] (bf16) x W[N, K]^T (bf16),   Mb <= 256
//
// A rollout decode step multiplies a few dozen to a few hundred token rows by
// every weight matrix of the model, so the product is bound by streaming W from
// HBM.  The kernel computes the TRANSPOSED product so that W supplies the
// 128-row MMA operand and the token rows are the (small) N side:
//
//   D^T[128 rows of W, NB] = W tile (A, K-major) x x (B, K-major),
//
// with NB = Mb rounded up to 16/32/64/128/256 (TMA fills the missing x rows with
// zeros).
//
// Work split: one CTA per (128-row tile of W, K range).  The S CTAs that share a
// tile (S in {1, 2, 4, 8}) form one thread-block cluster; each accumulates its K
// range in tensor memory, stores the fp32 partial tile into its own shared
// memory, and after a cluster barrier CTA s sums rows [s*128/S, (s+1)*128/S) of
// all S partials through distributed shared memory (ld.shared::cluster) and
// writes them as bf16.  No global workspace, no atomics, no second kernel, and
// the sum order is fixed (deterministic).  S is chosen on the host so that the
// grid holds about two CTAs per SM; each CTA keeps ~96 KB of its stream in
// flight (TMA ring), so the HBM pipe stays full even for the 32-50 MB matrices
// of one layer.
//
// Roles (6 warps): warp 0 = TMA producer (one lane; no multicast, every load
// reads this GPU's memory into this CTA's shared memory), warp 1 = tensor-memory
// allocator and MMA issuer (one lane), warps 2-5 = epilogue.  Every mbarrier
// wait is bounded: on expiry the kernel records an error code readable from the
// host (gemm_decode_error_flag), all roles leave their loops, and the CTA still
// takes part in both cluster barriers, frees its tensor memory and returns.
#include "tc_common.cuh"

#include <cstdlib>

namespace rlb {
namespace dec {

__device__ int g_dec_error = 0;

using namespace rlb::tc;

template <int NB>
struct DCfg {
  static constexpr int A_BYTES = BM * BK * 2;  // 128 x 64 W tile
  static constexpr int B_BYTES = NB * BK * 2;  // NB x 64 x tile
  static constexpr int RING_TARGET = 96 * 1024;
  static constexpr int STAGES_RAW = RING_TARGET / (A_BYTES + B_BYTES);
  static constexpr int STAGES = STAGES_RAW < 2 ? 2 : STAGES_RAW;
  static constexpr int RING = STAGES * (A_BYTES + B_BYTES);
  static constexpr int PART = BM * NB * 4;  // fp32 partial tile, token-major [NB][128]
  static constexpr int BODY = RING > PART ? RING : PART;
  static constexpr int SMEM = BODY + 1024 + 256;
  static constexpr uint32_t TMEM_COLS = NB < 32 ? 32 : NB;
  static constexpr uint32_t IDESC = idesc_bf16(BM, NB);
};

__device__ __forceinline__ uint32_t cl_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cl_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local_addr), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];\n" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

__device__ __forceinline__ bool dwait(uint32_t addr, uint32_t parity, volatile int* abort_flag, int code) {
  return mbar_wait_err(addr, parity, abort_flag, &g_dec_error, code);
}

template <int NB>
__global__ void __launch_bounds__(192, 2)
gemm_decode_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                   __nv_bfloat16* __restrict__ out, int Mb, int N, int K, int S, int kb_per) {
  using G = DCfg<NB>;
  constexpr int STAGES = G::STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * G::A_BYTES;
  float* part = reinterpret_cast<float*>(gbase);  // reuses the ring after the main loop
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + G::BODY);
  const uint32_t bar_full = smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_done = bar_empty + 8 * STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = S > 1 ? (int)cl_rank() : 0;
  const int tile = blockIdx.x / S;
  const int num_kb = (K + BK - 1) / BK;
  const int kb0 = split * kb_per;
  const int kb1 = min(num_kb, kb0 + kb_per);
  const int nkb = max(0, kb1 - kb0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(G::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_launch_dependents();
  if (warp == 0) {
    if (lane == 0) {
      // The weight does not depend on the kernel before this one: its first STAGES
      // tiles stream in while that kernel finishes (programmatic dependent launch);
      // the activation rows x are loaded only after pdl_wait().
      const int pre = min(nkb, STAGES);
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(bar_full + 8 * i, G::A_BYTES + G::B_BYTES);
        tma_load_2d(sA + i * G::A_BYTES, &tmap_w, bar_full + 8 * i, (kb0 + i) * BK, tile * BM);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sB + i * G::B_BYTES, &tmap_x, bar_full + 8 * i, (kb0 + i) * BK, 0);
      int j = pre;
      for (; j < nkb && !*abort_flag; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!dwait(bar_empty + 8 * s, ph ^ 1, abort_flag, 1)) break;
        mbar_expect_tx(bar_full + 8 * s, G::A_BYTES + G::B_BYTES);
        tma_load_2d(sA + s * G::A_BYTES, &tmap_w, bar_full + 8 * s, (kb0 + j) * BK, tile * BM);
        tma_load_2d(sB + s * G::B_BYTES, &tmap_x, bar_full + 8 * s, (kb0 + j) * BK, 0);
      }
      if (*abort_flag) {  // let the loads in flight land before the ring is reused or freed
        for (int i = max(0, j - STAGES); i < j; ++i) {
          const long long t0 = clock64();
          while (!mbar_test(bar_full + 8 * (i % STAGES), (i / STAGES) & 1) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = true;
      for (int j = 0; j < nkb; ++j) {
        const int s = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        if (!dwait(bar_full + 8 * s, ph, abort_flag, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = sA + s * G::A_BYTES, b0 = sB + s * G::B_BYTES;
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_bf16(tmem, desc_kmajor_sw128(a0 + k * 32), desc_kmajor_sw128(b0 + k * 32), G::IDESC,
                    (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(bar_empty + 8 * s);
      }
      if (ok && nkb > 0) umma_commit(bar_done);
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5: TMEM lanes quad*32.. = W rows; columns = token rows.  They
    // write `out`, which may reuse memory an earlier kernel still reads: wait for it.
    pdl_wait();
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int n = tile * BM + row;
    bool have = nkb > 0;
    if (have) {
      have = dwait(bar_done, 0, abort_flag, 3);
      tc_fence_after();
    }
#pragma unroll 1
    for (int c = 0; c < NB / 32 || (NB < 32 && c == 0); ++c) {
      uint32_t r[32];
      if (have) tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + c * 32, r);
      const int ncol = NB < 32 ? NB : 32;
      if (S == 1) {
        if (n < N) {
          for (int t = 0; t < ncol; ++t) {
            const int m = c * 32 + t;
            if (m < Mb) out[(long long)m * N + n] = __float2bfloat16_rn(have ? __uint_as_float(r[t]) : 0.f);
          }
        }
      } else {
        for (int t = 0; t < ncol; ++t) part[(c * 32 + t) * BM + row] = have ? __uint_as_float(r[t]) : 0.f;
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (S > 1) {
    cl_sync();  // every split's partial is in its shared memory
    const int R = BM / S;
    const uint32_t pbase = smem_u32(part);
    for (int e = threadIdx.x; e < R * Mb; e += blockDim.x) {
      const int m = e / R;
      const int row = split * R + (e % R);
      const int n = tile * BM + row;
      if (n >= N) continue;
      float acc = 0.f;
      for (int s = 0; s < S; ++s) acc += ld_cluster_f32(pbase + (uint32_t)((m * BM + row) * 4), (uint32_t)s);
      out[(long long)m * N + n] = __float2bfloat16_rn(acc);
    }
    cl_sync();  // no CTA leaves while a peer may still read its partial
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(G::TMEM_COLS));
  }
}

}  // namespace dec
}  // namespace rlb

using namespace rlb;

namespace {

// RL_B200_DECODE_PDL=0 turns the early launch off (for A/B timing).
bool dec_pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("RL_B200_DECODE_PDL");
    on = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return on == 1;
}

CUtensorMap dec_tmap(const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "rl_b200 gemm_decode: cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

template <int NB>
void launch_decode(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, int Mb, int N, int K, int S) {
  using G = dec::DCfg<NB>;
  const CUtensorMap tw = dec_tmap(w.data_ptr(), N, K, tc::BM);
  const CUtensorMap tx = dec_tmap(x.data_ptr(), Mb, K, NB);
  auto kern = dec::gemm_decode_kernel<NB>;
  RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
  const int tiles = (N + tc::BM - 1) / tc::BM;
  const int num_kb = (K + tc::BK - 1) / tc::BK;
  const int kb_per = (num_kb + S - 1) / S;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles * S);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = stream();
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // programmatic dependent launch (see the producer): may start before the previous
  // kernel on the stream has finished
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = dec_pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  RLB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tw, tx, (__nv_bfloat16*)out.data_ptr(), Mb, N, K, S, kb_per));
}

}  // namespace

// out [Mb, N] = x [Mb, K] @ w [N, K]^T for Mb <= 256 (decode batches).
//   splits: 0 = choose (about two CTAs per SM), else 1, 2, 4 or 8.
at::Tensor gemm_decode_split(at::Tensor x, at::Tensor w, int64_t splits) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "rl_b200 gemm_decode: bf16 CUDA operands expected");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "rl_b200 gemm_decode: x [M,K], w [N,K]");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous(), "rl_b200 gemm_decode: contiguous operands");
  const int Mb = x.size(0), N = w.size(0), K = x.size(1);
  TORCH_CHECK(Mb >= 1 && Mb <= 256, "rl_b200 gemm_decode: 1 <= rows <= 256");
  TORCH_CHECK(K % 8 == 0 && K > 0, "rl_b200 gemm_decode: K must be a positive multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "rl_b200 gemm_decode: 16-byte aligned operands");
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty({Mb, N}, x.options());
  if (N == 0) return out;
  const int tiles = (N + tc::BM - 1) / tc::BM;
  const int num_kb = (K + tc::BK - 1) / tc::BK;
  int S = (int)splits;
  if (S <= 0) {
    const int target = 2 * num_sms();
    S = 1;
    while (S < 8 && tiles * S * 2 <= target && (S * 2) <= num_kb) S *= 2;
  }
  TORCH_CHECK(S == 1 || S == 2 || S == 4 || S == 8, "rl_b200 gemm_decode: splits must be 1, 2, 4 or 8");
  TORCH_CHECK(S <= num_kb, "rl_b200 gemm_decode: more splits than 64-wide K blocks");
  if (Mb <= 16) launch_decode<16>(x, w, out, Mb, N, K, S);
  else if (Mb <= 32) launch_decode<32>(x, w, out, Mb, N, K, S);
  else if (Mb <= 64) launch_decode<64>(x, w, out, Mb, N, K, S);
  else if (Mb <= 128) launch_decode<128>(x, w, out, Mb, N, K, S);
  else launch_decode<256>(x, w, out, Mb, N, K, S);
  return out;
}

at::Tensor gemm_decode(at::Tensor x, at::Tensor w) { return gemm_decode_split(x, w, 0); }

int64_t gemm_decode_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, dec::g_dec_error, sizeof(int)));
  if (reset) {
    int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(dec::g_dec_error, &z, sizeof(int)));
  }
  return v;
}
