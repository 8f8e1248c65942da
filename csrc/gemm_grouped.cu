// Grouped (per-expert) bf16 GEMM for MoE layers on the 5th-generation tensor
// cores (sm_100a):
//
//   Y[r, :] = X[r, :] . W[e]^T   for every row r in expert e's segment
//             [offs[e-1], offs[e])   (offs = inclusive prefix sum of the counts)
//
// X [T, K] bf16 (rows grouped by expert), W [E, N, K] bf16, Y [T, N] bf16.
// The tile schedule is built on the device from ``offs`` (no host read of the
// per-expert counts): every CTA turns the counts into per-expert tile counts and
// their prefix sums in shared memory, then walks the global tile index in a
// persistent loop (tile -> expert by binary search).  An expert's m-tiles start
// at its first row, so a tile may overhang into the next expert's rows: those
// rows are computed but not stored.  W is addressed as a 2-D [E * N, K] tensor;
// N must be a multiple of the tile width so that no B tile crosses experts.
//
// Pipeline as in the dense kernel (warp 0 TMA, warp 1 TMEM + MMA issue, warps
// 2-5 epilogue, double-buffered TMEM accumulators, bounded mbarrier waits, no
// multicast).
#include "tc_common.cuh"

namespace rlb {
namespace gg {

using namespace tc;
__device__ int g_gg_error = 0;
constexpr int MAX_E = 512;

__device__ __forceinline__ bool wait(uint32_t addr, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_err(addr, parity, abort_flag, &g_gg_error, 1);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
grouped_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               const int* __restrict__ offs, __nv_bfloat16* __restrict__ C, int N, int K, int E) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16(BM, BN);
  __shared__ int s_tile0[MAX_E + 1];  // first global tile of expert e
  __shared__ int s_row0[MAX_E + 1];   // first row of expert e
  extern __shared__ uint8_t smem_raw[];
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
  const int num_n = N / BN;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    int tiles = 0, prev = 0;
    for (int e = 0; e < E; ++e) {
      const int end = offs[e];
      s_tile0[e] = tiles;
      s_row0[e] = prev;
      tiles += ((end - prev + BM - 1) / BM) * num_n;
      prev = end;
    }
    s_tile0[E] = tiles;
    s_row0[E] = prev;
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
  const int num_tiles = s_tile0[E];

  // global tile -> (expert, first row of the tile, end row of the expert, n-tile)
  auto coords = [&](int tile, int& e, int& row0, int& row_end, int& nt) {
    int lo = 0, hi = E - 1;
    while (lo < hi) {  // last expert whose first tile <= tile (empty experts share the next one's)
      const int mid = (lo + hi + 1) >> 1;
      if (s_tile0[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    e = lo;
    const int local = tile - s_tile0[e];
    row0 = s_row0[e] + (local / num_n) * BM;
    row_end = s_row0[e + 1];
    nt = local % num_n;
  };

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok && !*abort_flag; tile += gridDim.x) {
        int e, row0, row_end, nt;
        coords(tile, e, row0, row_end, nt);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(bar_full + 8 * s, A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmap_a, bar_full + 8 * s, kb * BK, row0);
          tma_load_2d(sB + s * B_BYTES, &tmap_b, bar_full + 8 * s, kb * BK, e * N + nt * BN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        if (!wait(bar_tempty + 8 * acc, ((local >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait(bar_full + 8 * s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + s * A_BYTES, b0 = sB + s * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(tmem_d, desc_kmajor_sw128(a0 + k * 32), desc_kmajor_sw128(b0 + k * 32), IDESC,
                      (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(bar_empty + 8 * s);
        }
        if (!ok) break;
        umma_commit(bar_tfull + 8 * acc);
      }
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int e, row0, row_end, nt;
      coords(tile, e, row0, row_end, nt);
      const int acc = local & 1;
      if (!wait(bar_tfull + 8 * acc, (local >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      const int m = row0 + row_in_tile;
      const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + c * 32, r);
        if (m < row_end) {
          __nv_bfloat16* dst = C + (long long)m * N + nt * BN + c * 32;
          uint4 v[4];
          uint32_t* pv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
            pv[j] = *reinterpret_cast<uint32_t*>(&h);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = v[j];
        }
      }
      tc_fence_before();
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

template <int BN, int STAGES>
void launch(const at::Tensor& x, const at::Tensor& w, const at::Tensor& offs, at::Tensor& y) {
  const int T = x.size(0), K = x.size(1), E = w.size(0), N = w.size(1);
  const CUtensorMap ta = make_tmap_2d(x.data_ptr(), T, K, BM);
  const CUtensorMap tb = make_tmap_2d(w.data_ptr(), (int64_t)E * N, K, BN);
  const int smem = STAGES * (BM * BK * 2 + BN * BK * 2) + 1024 + 256;
  auto kern = grouped_kernel<BN, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  // tiles are counted on the device; an upper bound sizes the grid
  const long long max_tiles = ((long long)(T + BM - 1) / BM + E) * (N / BN);
  const int grid = (int)std::min<long long>(max_tiles, num_sms());
  kern<<<grid, 192, smem, stream()>>>(ta, tb, offs.data_ptr<int>(), (__nv_bfloat16*)y.data_ptr(), N, K, E);
  RLB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace gg
}  // namespace rlb

using namespace rlb;

// x [T, K] bf16 rows grouped by expert, w [E, N, K] bf16, offs int32 [E]
// (inclusive prefix sum of the per-expert row counts, offs[E-1] == T).
at::Tensor grouped_gemm_nt(at::Tensor x, at::Tensor w, at::Tensor offs) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && offs.is_cuda(), "rl_b200 grouped_gemm_nt: CUDA tensors expected");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && offs.scalar_type() == at::kInt,
              "rl_b200 grouped_gemm_nt: bf16 x / w and int32 offsets expected");
  TORCH_CHECK(x.dim() == 2 && w.dim() == 3 && w.size(2) == x.size(1) && offs.numel() == w.size(0) &&
                  x.is_contiguous() && w.is_contiguous() && offs.is_contiguous(),
              "rl_b200 grouped_gemm_nt: x [T, K], w [E, N, K], offs [E], contiguous");
  const int K = x.size(1), E = w.size(0), N = w.size(1);
  TORCH_CHECK(E >= 1 && E <= gg::MAX_E, "rl_b200 grouped_gemm_nt: 1..512 experts");
  TORCH_CHECK(K % 64 == 0 && N % 128 == 0, "rl_b200 grouped_gemm_nt: K % 64 == 0 and N % 128 == 0 required");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "rl_b200 grouped_gemm_nt: 16-byte aligned operands");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = at::empty({x.size(0), N}, x.options());
  if (x.size(0) == 0) return y;
  if (N % 256 == 0) gg::launch<256, 4>(x, w, offs, y);
  else gg::launch<128, 6>(x, w, offs, y);
  return y;
}

int64_t grouped_gemm_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, gg::g_gg_error, sizeof(int)));
  if (reset) {
    int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(gg::g_gg_error, &z, sizeof(int)));
  }
  return v;
}
