// Persistent bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M, N] (bf16) = A[M, K] (bf16, row-major) x B[N, K]^T (bf16, row-major)
//
// Structure (one CTA per SM, 6 warps):
//   warp 0      TMA producer: one elected lane issues cp.async.bulk.tensor loads
//               of 128x64 A tiles and BNx64 B tiles (128-byte swizzle) into a
//               STAGES-deep shared-memory ring, signalling mbarriers with the
//               transaction byte count.  No multicast: every CTA loads its own
//               tiles (this kernel is also the template for the peer-memory
//               variants that run on several GPUs).
//   warp 1      allocates 2*BN tensor-memory columns (two accumulators), then
//               one lane issues tcgen05.mma (M=128, N=BN, K=16) per 16-wide K
//               slice, committing each stage back to the producer and each
//               finished tile to the epilogue.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns at a time from the
//               accumulator their warp may access (TMEM lane quadrant = warp % 4),
//               convert to bf16 and store; then release the accumulator so the
//               MMA warp can start the tile after next.
// Tiles are visited in a grouped raster (GROUP_M m-tiles per column sweep) for
// L2 reuse.  Every mbarrier wait is bounded in time: on expiry the kernel sets
// an error word (readable from the host), raises a CTA-wide abort flag so all
// roles drain, frees its tensor memory and returns.
#include "tc_common.cuh"

namespace rlb {
namespace tc {

__device__ int g_error = 0;

constexpr int GROUP_M = 8;

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mt, int& nt) {
  const int group = GROUP_M * num_n;
  const int gid = tile / group;
  const int first_m = gid * GROUP_M;
  const int gsize = min(num_m - first_m, GROUP_M);
  const int in = tile % group;
  mt = first_m + in % gsize;
  nt = in / gsize;
}

// Bounded wait on this file's error word.
__device__ __forceinline__ bool mbar_wait(uint32_t addr, uint32_t parity, volatile int* abort_flag) {
  return mbar_wait_err(addr, parity, abort_flag, &g_error, 1);
}

// ------------------------------------------------------------------------
// Fused reduce-scatter epilogue (tensor-parallel row-parallel linear with
// sequence parallelism).  Each of `n` ranks computes the full partial product
// P_r = A_r B_r^T ([M, N]); rank d owns output rows [d*Ms, (d+1)*Ms) of
// sum_r P_r.  Tiles are scheduled destination-major starting with the next
// rank, own tiles last.  A tile for rank d != me is converted to bf16 and
// stored straight into d's receive buffer (slot `me`) over NVLink, then a
// release flag (value = epoch) is set in d's flag array.  An own tile waits
// (acquire, bounded) for every peer's flag, adds the received partials to its
// fp32 accumulator and writes the final rows.
//
// Flow control: receive slots and flags are double-buffered by epoch parity p.
// When the LAST CTA of a rank's launch for epoch e finishes (grid-wide counter),
// that rank has consumed everything it received for e and acknowledges it to
// every producer (one word per parity and consumer, in the producer's memory).
// Before its first store of epoch e a producer waits for the destination's
// acknowledgement of epoch e - 2 (same parity slot).  The acknowledgement is
// per launch, not per tile, so row counts may change from call to call.
struct RSArgs {
  int n, me, Ms;
  uint32_t epoch;
  __nv_bfloat16* recv[8];   // per rank: [2][n][Ms][N] bf16 (peer pointers; recv[me] is local)
  uint32_t* flags[8];       // per rank: [2][n][tiles_per_shard] u32 (data-ready, written by producers)
  uint32_t* acks[8];        // per rank: [2][n] u32 slot-free words (written by consumers) + [2] local counters
  __nv_bfloat16* out;       // this rank's [Ms, N] output
  // all-gather -> GEMM (EPI == 2): A is the gathered [n*Ms, K] input whose shard j
  // is ready once shard_flags[j] >= epoch; tiles visit the own shard first, then
  // the others in ring order (the order their copies land)
  const uint32_t* shard_flags;
  long long wait;  // bound of every wait on a peer's flag or a copy-engine flag (cycles)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= epoch (unsigned, epochs increase).  false on expiry.
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t epoch, volatile int* abort_flag,
                                          long long limit) {
  const long long t0 = clock64();
  while ((int)(ld_acquire_sys(p) - epoch) < 0) {
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      atomicExch(&g_error, 2);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void rs_tile_coords(int tile, int num_n, int mts, const RSArgs& rs, int& dest, int& mt,
                                               int& nt, int& within) {
  const int per = mts * num_n;
  const int j = tile / per;
  within = tile % per;
  dest = (rs.me + 1 + j) % rs.n;
  mt = dest * mts + within / num_n;
  nt = within % num_n;
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(192, 1)
gemm_nt_kernel_t(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 __nv_bfloat16* __restrict__ C, int M, int N, int K, const __grid_constant__ RSArgs rs) {
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = idesc_bf16(BM, BN);
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
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int mts = (EPI == 1) ? rs.Ms / BM : 0;  // m-tiles per destination shard
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  // tile -> (m-tile, n-tile); for the reduce-scatter epilogue also (dest, index within shard)
  auto coords = [&](int tile, int& mt, int& nt, int& dest, int& within) {
    if constexpr (EPI == 1) {
      rs_tile_coords(tile, num_n, mts, rs, dest, mt, nt, within);
    } else if constexpr (EPI == 2) {
      int mo;
      tile_coords(tile, num_m, num_n, mo, nt);
      const int per = rs.Ms / BM;
      dest = (rs.me + mo / per) % rs.n;  // source shard of this m-tile
      mt = dest * per + mo % per;
      within = 0;
    } else {
      tile_coords(tile, num_m, num_n, mt, nt);
      dest = 0;
      within = 0;
    }
  };

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
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int mt, nt, dest, within;
        coords(tile, mt, nt, dest, within);
        if constexpr (EPI == 2) {
          // the copy engine lands shard `dest` and then writes its flag (stream
          // memory op); order the TMA reads of that shard after the flag
          if (!wait_flag(rs.shard_flags + dest, rs.epoch, abort_flag, rs.wait)) break;
          asm volatile("fence.proxy.async.global;\n" ::: "memory");
        }
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) break;
          mbar_expect_tx(bar_full + 8 * s, A_BYTES + B_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmap_a, bar_full + 8 * s, kb * BK, mt * BM);
          tma_load_2d(sB + s * B_BYTES, &tmap_b, bar_full + 8 * s, kb * BK, nt * BN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(bar_tempty + 8 * acc, aph ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(bar_full + 8 * s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + s * A_BYTES, b0 = sB + s * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16(tmem_d, desc_kmajor_sw128(a0 + k * 32), desc_kmajor_sw128(b0 + k * 32), IDESC,
                      (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(bar_empty + 8 * s);
        }
        if (!ok) break;
        umma_commit(bar_tfull + 8 * acc);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      int mt, nt, dest, within;
      coords(tile, mt, nt, dest, within);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!mbar_wait(bar_tfull + 8 * acc, aph, abort_flag)) break;
      tc_fence_after();
      const int m = mt * BM + row_in_tile;
      const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
      if constexpr (EPI == 1) {
        const int row_s = m - dest * rs.Ms;  // row inside the destination shard
        const int tiles_per_shard = mts * num_n;
        const int par = (int)(rs.epoch & 1u);
        if (dest != rs.me) {
          // partial tile -> peer's receive slot `me`, then a release flag; first make
          // sure the peer consumed what this slot held two epochs ago
          wait_flag(rs.acks[rs.me] + par * rs.n + dest, rs.epoch - 2u, abort_flag, rs.wait);
          __nv_bfloat16* dst_base = rs.recv[dest] + (((long long)par * rs.n + rs.me) * rs.Ms + row_s) * N;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(trow + c * 32, r);
            const int n0 = nt * BN + c * 32;
            if (n0 < N) {
              uint4 v[4];
              uint32_t* pv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                pv[j] = *reinterpret_cast<uint32_t*>(&h);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst_base + n0)[j] = v[j];
            }
          }
          __threadfence_system();
          tc_fence_before();
          asm volatile("bar.sync 1, 128;\n" ::: "memory");
          if (warp == 2 && lane == 0)
            st_release_sys(rs.flags[dest] + ((long long)par * rs.n + rs.me) * tiles_per_shard + within, rs.epoch);
        } else {
          // own tile: wait for every peer's partial, reduce, write the final rows
          bool ok = true;
          for (int src = 0; src < rs.n && ok; ++src)
            if (src != rs.me)
              ok = wait_flag(rs.flags[rs.me] + ((long long)par * rs.n + src) * tiles_per_shard + within, rs.epoch,
                             abort_flag, rs.wait);
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(trow + c * 32, r);
            const int n0 = nt * BN + c * 32;
            if (n0 >= N) continue;
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
            if (ok) {
              for (int src = 0; src < rs.n; ++src) {
                if (src == rs.me) continue;
                const uint4* pr = reinterpret_cast<const uint4*>(
                    rs.recv[rs.me] + (((long long)par * rs.n + src) * rs.Ms + row_s) * N + n0);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  uint4 u = pr[q];
                  const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    float2 t2 = __bfloat1622float2(hb[e]);
                    f[q * 8 + 2 * e] += t2.x;
                    f[q * 8 + 2 * e + 1] += t2.y;
                  }
                }
              }
            }
            uint4 v[4];
            uint32_t* pv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
              pv[j] = *reinterpret_cast<uint32_t*>(&h);
            }
            __nv_bfloat16* dst = rs.out + (long long)row_s * N + n0;
#pragma unroll
            for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = v[j];
          }
          tc_fence_before();
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + c * 32, r);
          const int n0 = nt * BN + c * 32;
          if (m < M && n0 < N) {
            __nv_bfloat16* dst = C + (long long)m * N + n0;
            if (n0 + 32 <= N && (N % 8) == 0) {
              uint4 v[4];
              uint32_t* pv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
                pv[j] = *reinterpret_cast<uint32_t*>(&h);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = v[j];
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n0 + j < N) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
            }
          }
        }
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_tempty + 8 * acc);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (EPI == 1) {
    if (threadIdx.x == 0) {
      // last CTA out acknowledges epoch e to every producer (slots of parity e&1 are free)
      const int par = (int)(rs.epoch & 1u);
      uint32_t* counter = rs.acks[rs.me] + 2 * rs.n + par;
      __threadfence();
      const uint32_t prev = atomicAdd(counter, 1u);
      if (prev == gridDim.x - 1) {
        *counter = 0u;
        __threadfence_system();
        for (int src = 0; src < rs.n; ++src)
          if (src != rs.me) st_release_sys(rs.acks[src] + par * rs.n + rs.me, rs.epoch);
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

}  // namespace tc
}  // namespace rlb

using namespace rlb;

template <int BN, int STAGES, int EPI>
static void launch_gemm(const at::Tensor& a, const at::Tensor& b, __nv_bfloat16* c, int M, int N, int K,
                        const tc::RSArgs& rs) {
  const CUtensorMap ta = make_tmap_2d(a.data_ptr(), M, K, tc::BM);
  const CUtensorMap tb = make_tmap_2d(b.data_ptr(), N, K, BN);
  const int smem = STAGES * (tc::BM * tc::BK * 2 + BN * tc::BK * 2) + 1024 + 256;
  auto kern = tc::gemm_nt_kernel_t<BN, STAGES, EPI>;
  RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int tiles = ((M + tc::BM - 1) / tc::BM) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms());
  kern<<<grid, 192, smem, stream()>>>(ta, tb, c, M, N, K, rs);
  RLB_CUDA_CHECK(cudaGetLastError());
}

at::Tensor gemm_nt(at::Tensor a, at::Tensor b) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "rl_b200 gemm_nt: bf16 CUDA operands expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "rl_b200 gemm_nt: a [M,K], b [N,K]");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous(), "rl_b200 gemm_nt: operands must be contiguous");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(K % 8 == 0 && K > 0, "rl_b200 gemm_nt: K must be a positive multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "rl_b200 gemm_nt: operands must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(a.device());
  auto c = at::empty({M, N}, a.options());
  if (M == 0 || N == 0) return c;
  tc::RSArgs none{};
  none.wait = peer_wait_cycles();
  if (N >= 256) launch_gemm<256, 4, 0>(a, b, (__nv_bfloat16*)c.data_ptr(), M, N, K, none);
  else launch_gemm<128, 6, 0>(a, b, (__nv_bfloat16*)c.data_ptr(), M, N, K, none);
  return c;
}

// Fused GEMM + reduce-scatter over `n` ranks of one node (see RSArgs).
//   a [M, K_local], b [N, K_local] (this rank's K shard), out [M/n, N] (bf16).
//   recv_ptrs / flag_ptrs / ack_ptrs: device addresses of every rank's symmetric
//   receive buffer ([2][n][M/n][N] bf16), flag array ([2][n][(M/n/128) *
//   ceil(N/BN)] u32) and ack words ([2][n] + [2] counters, u32); all zeroed once.
// Every rank must launch with the same epoch; epochs increase per call.
void gemm_rs(at::Tensor a, at::Tensor b, at::Tensor out, std::vector<int64_t> recv_ptrs,
             std::vector<int64_t> flag_ptrs, std::vector<int64_t> ack_ptrs, int64_t me, int64_t epoch) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "rl_b200 gemm_rs: bf16 CUDA operands expected");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.is_contiguous(), "rl_b200 gemm_rs: contiguous operands");
  const int n = (int)recv_ptrs.size();
  TORCH_CHECK(n >= 1 && n <= 8 && (int)flag_ptrs.size() == n && (int)ack_ptrs.size() == n && me >= 0 && me < n,
              "rl_b200 gemm_rs: bad rank set");
  TORCH_CHECK(epoch >= 1, "rl_b200 gemm_rs: epochs start at 1");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(M % (n * tc::BM) == 0, "rl_b200 gemm_rs: M must be a multiple of 128 * ranks");
  TORCH_CHECK(N % 32 == 0 && K % 8 == 0, "rl_b200 gemm_rs: N % 32 == 0 and K % 8 == 0 required");
  TORCH_CHECK(out.size(0) == M / n && out.size(1) == N, "rl_b200 gemm_rs: out must be [M/n, N]");
  const c10::cuda::CUDAGuard guard(a.device());
  tc::RSArgs rs{};
  rs.wait = peer_wait_cycles();
  rs.n = n;
  rs.me = (int)me;
  rs.Ms = M / n;
  rs.epoch = (uint32_t)epoch;
  for (int i = 0; i < n; ++i) {
    rs.recv[i] = reinterpret_cast<__nv_bfloat16*>((uintptr_t)recv_ptrs[i]);
    rs.flags[i] = reinterpret_cast<uint32_t*>((uintptr_t)flag_ptrs[i]);
    rs.acks[i] = reinterpret_cast<uint32_t*>((uintptr_t)ack_ptrs[i]);
  }
  rs.out = (__nv_bfloat16*)out.data_ptr();
  if (N >= 256) launch_gemm<256, 4, 1>(a, b, nullptr, M, N, K, rs);
  else launch_gemm<128, 6, 1>(a, b, nullptr, M, N, K, rs);
}

int64_t gemm_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, tc::g_error, sizeof(int)));
  if (reset) {
    int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(tc::g_error, &z, sizeof(int)));
  }
  return v;
}

// All-gather -> GEMM: out [M, N] = gathered [M, K] x b [N, K]^T where the rows of
// shard j (M / n rows each) become valid when shard_flags[j] >= epoch.  The
// gathered rows are written by copy-engine transfers from the peers' symmetric
// buffers on a side stream (rl_b200/parallel/fused.py), each followed by a
// stream write of its shard flag; the kernel starts on the own shard at once
// and waits (bounded) per remote shard, so the transfers overlap the MMA work.
at::Tensor gemm_ag(at::Tensor a, at::Tensor b, at::Tensor shard_flags, int64_t n, int64_t me, int64_t epoch) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "rl_b200 gemm_ag: bf16 CUDA operands expected");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && a.size(1) == b.size(1), "rl_b200 gemm_ag: a [M,K], b [N,K]");
  TORCH_CHECK(shard_flags.is_cuda() && shard_flags.scalar_type() == at::kInt && shard_flags.numel() >= n,
              "rl_b200 gemm_ag: int32 shard flags on the device");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(n >= 1 && n <= 8 && me >= 0 && me < n && M % (n * tc::BM) == 0,
              "rl_b200 gemm_ag: M must be a multiple of 128 * ranks");
  TORCH_CHECK(K % 8 == 0 && epoch >= 1, "rl_b200 gemm_ag: K % 8 == 0, epoch >= 1");
  const c10::cuda::CUDAGuard guard(a.device());
  auto c = at::empty({M, N}, a.options());
  tc::RSArgs ag{};
  ag.wait = peer_wait_cycles();
  ag.n = (int)n;
  ag.me = (int)me;
  ag.Ms = M / (int)n;
  ag.epoch = (uint32_t)epoch;
  ag.shard_flags = reinterpret_cast<const uint32_t*>(shard_flags.data_ptr<int>());
  if (N >= 256) launch_gemm<256, 4, 2>(a, b, (__nv_bfloat16*)c.data_ptr(), M, N, K, ag);
  else launch_gemm<128, 6, 2>(a, b, (__nv_bfloat16*)c.data_ptr(), M, N, K, ag);
  return c;
}

// Stream memory write of a 32-bit word (executed by the stream front end, no
// kernel): signals data landed by an earlier copy on the same stream.
void stream_write_u32(int64_t ptr, int64_t value) {
  static PFN_cuStreamWriteValue32_v11070 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    RLB_CUDA_CHECK(cudaGetDriverEntryPointByVersion("cuStreamWriteValue32", &p, 11070, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "rl_b200: cuStreamWriteValue32 unavailable");
    fn = reinterpret_cast<PFN_cuStreamWriteValue32_v11070>(p);
  }
  CUresult r = fn(reinterpret_cast<CUstream>(stream()), (CUdeviceptr)ptr, (cuuint32_t)value, 0);
  TORCH_CHECK(r == CUDA_SUCCESS, "rl_b200: cuStreamWriteValue32 failed (", (int)r, ")");
}
