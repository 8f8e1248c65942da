// Block-scaled e4m3 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M, N] (bf16) = sum_kb  sa[m, kb] * sb[n / 128, kb] * (A[m, kb-block] . B[n, kb-block])
//
// A [M, K] e4m3 activations with one fp32 scale per row and 128-wide K block
// (1 x 128), B [N, K] e4m3 weights with one fp32 scale per 128 x 128 block,
// K a multiple of 128.  The scales are arbitrary fp32 values (not only powers
// of two), so they cannot ride on the MMA's hardware block scaling: every
// 128-wide K block is multiplied by tcgen05.mma kind::f8f6f4 (4 instructions of
// K = 32) into its OWN tensor-memory accumulator, and the epilogue warps read
// it back, scale it and add it to fp32 accumulators held in registers
// ("promotion").  Four 128-column TMEM buffers let the MMAs of the next blocks
// run while earlier blocks are promoted.
//
// One CTA per SM, 10 warps:
//   warp 0      TMA producer (128 x 128-byte tiles of A and B, 128-byte
//               swizzle, STAGES-deep ring; no multicast);
//   warp 1      TMEM allocation (512 columns) and the MMA issuer;
//   warps 2-9   promotion / epilogue: warp w owns TMEM lanes 32 * (w % 4) ..
//               +31 (= tile rows) and columns 64 * ((w - 2) / 4) .. +63.
// Small-M shapes (decode) split K over CTAs (`splits`): each split adds its
// partial tile into an fp32 workspace with atomics; the host casts it.
// Every mbarrier wait is bounded (error word + CTA abort flag, TMEM freed).
#include "tc_common.cuh"

namespace rlb {
namespace f8 {

using tc::BM;
__device__ int g_f8_error = 0;

constexpr int BN = 128;
constexpr int KB = 128;   // K block = scale block = one 128-byte swizzle row
constexpr int NBUF = 4;   // TMEM accumulators (NBUF * BN columns)
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
// D = f32 (bits 4-5), A = B = e4m3 (bits 7-9, 10-12 zero), K-major, N >> 3, M >> 4
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate));
}

__device__ __forceinline__ bool wait(uint32_t addr, uint32_t parity, volatile int* abort_flag) {
  return tc::mbar_wait_err(addr, parity, abort_flag, &g_f8_error, 1);
}

// work unit -> (m-tile, n-tile, first and end K block); grouped raster for L2 reuse
__device__ __forceinline__ void unit_coords(int u, int num_m, int num_n, int splits, int kper, int num_kb, int& mt,
                                            int& nt, int& kb0, int& kb1) {
  const int split = u % splits;
  const int t = u / splits;
  constexpr int G = 8;
  const int group = G * num_n;
  const int first_m = (t / group) * G;
  const int gsize = min(num_m - first_m, G);
  const int in = t % group;
  mt = first_m + in % gsize;
  nt = in / gsize;
  kb0 = split * kper;
  kb1 = min(num_kb, kb0 + kper);
}

template <int STAGES>
__global__ void __launch_bounds__(THREADS, 1)
gemm_f8_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               const float* __restrict__ sa, const float* __restrict__ sb, __nv_bfloat16* __restrict__ C,
               float* __restrict__ C32, int M, int N, int K, int splits, int kper) {
  constexpr int A_BYTES = BM * KB;
  constexpr int B_BYTES = BN * KB;
  constexpr uint32_t TMEM_COLS = NBUF * BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + STAGES * (A_BYTES + B_BYTES));
  const uint32_t bar_full = tc::smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  const uint32_t bar_tfull = bar_empty + 8 * STAGES;
  const uint32_t bar_tempty = bar_tfull + 8 * NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 2 * NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int num_kb = K / KB;
  const int num_units = num_m * num_n * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(bar_full + 8 * s, 1);
      tc::mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      tc::mbar_init(bar_tfull + 8 * b, 1);
      tc::mbar_init(bar_tempty + 8 * b, EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tc::smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok && !*abort_flag; u += gridDim.x) {
        int mt, nt, kb0, kb1;
        unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc::mbar_expect_tx(bar_full + 8 * s, A_BYTES + B_BYTES);
          tc::tma_load_2d(sA + s * A_BYTES, &tmap_a, bar_full + 8 * s, kb * KB, mt * BM);
          tc::tma_load_2d(sB + s * B_BYTES, &tmap_b, bar_full + 8 * s, kb * KB, nt * BN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, j = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok && !*abort_flag; u += gridDim.x) {
        int mt, nt, kb0, kb1;
        unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it, ++j) {
          const int buf = j % NBUF;
          const uint32_t bph = (j / NBUF) & 1;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait(bar_tempty + 8 * buf, bph ^ 1, abort_flag) || !wait(bar_full + 8 * s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a0 = sA + s * A_BYTES, b0 = sB + s * B_BYTES;
          const uint32_t tmem_d = tmem_base + buf * BN;
#pragma unroll
          for (int k = 0; k < KB / 32; ++k)
            umma_f8(tmem_d, tc::desc_kmajor_sw128(a0 + k * 32), tc::desc_kmajor_sw128(b0 + k * 32), k > 0 ? 1u : 0u);
          tc::umma_commit(bar_empty + 8 * s);
          tc::umma_commit(bar_tfull + 8 * buf);
        }
      }
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16) + half * 64;
    int j = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int mt, nt, kb0, kb1;
      unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
      const int m = mt * BM + row_in_tile;
      const bool row_ok = m < M;
      const float* sa_row = sa + (long long)(row_ok ? m : 0) * num_kb;
      const float* sb_row = sb + (long long)nt * num_kb;
      float acc[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) acc[c] = 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++j) {
        const int buf = j % NBUF;
        const uint32_t bph = (j / NBUF) & 1;
        const float sc = row_ok ? sa_row[kb] * sb_row[kb] : 0.f;
        if (!wait(bar_tfull + 8 * buf, bph, abort_flag)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tc::tmem_ld32(lane_base + buf * BN + c * 32, r);
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[c * 32 + e] = fmaf(sc, __uint_as_float(r[e]), acc[c * 32 + e]);
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_tempty + 8 * buf);
      }
      if (!ok || !row_ok) continue;
      const int n0 = nt * BN + half * 64;
      if (splits == 1) {
        __nv_bfloat16* dst = C + (long long)m * N + n0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (n0 + q * 8 < N) {
            uint4 v;
            uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 h = __floats2bfloat162_rn(acc[q * 8 + 2 * e], acc[q * 8 + 2 * e + 1]);
              pv[e] = *reinterpret_cast<uint32_t*>(&h);
            }
            *reinterpret_cast<uint4*>(dst + q * 8) = v;
          }
        }
      } else {
        float* dst = C32 + (long long)m * N + n0;
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (n0 + c < N) atomicAdd(dst + c, acc[c]);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// Power-of-two scales: the tensor cores apply them.  tcgen05.mma
// kind::mxf8f6f4.block_scale multiplies each 32-wide K slice of A row m by
// 2^(e_a[m] - 127) and of B column n by 2^(e_b[n] - 127) (UE8M0 scale bytes
// read from tensor memory), so one accumulator runs over all of K and no
// promotion is needed.  A 1 x 128 / 128 x 128 block scale is the same byte
// for the four K slices of a 128-wide block.
//
// Tensor-memory layout of the scale factors (one slot of 16 columns per
// pipeline stage): the scale of row r (A: 0..127, B: 0..BN-1) sits in column
// slot + r / 32 (A) or slot + 8 + r / 32 (B), lane r % 32 of EVERY 32-lane
// quadrant (replicated four times), byte 0 of the 32-bit word (the MMA's scale
// factor id selects the byte).
//
// 128 x 224 tiles: two 224-column accumulators (448 columns) plus four 16-column
// scale slots fill the 512 columns of tensor memory, so the epilogue of one
// tile overlaps the main loop of the next.  10 warps: 0 TMA, 1 MMA, 2-5
// epilogue, 6-9 write each stage's scale bytes (tcgen05.st) once the MMAs that
// read the slot before have completed.
constexpr int MX_BN = 224;
constexpr int MX_STAGES = 4;
constexpr uint32_t MX_SF_COL = 2 * MX_BN;  // 448
// block-scaled descriptor: A = B = e4m3, K-major, N >> 3, scale format UE8M0 (bit 23), M >> 4, sf ids 0
constexpr uint32_t MX_IDESC = ((uint32_t)(MX_BN >> 3) << 17) | (1u << 23) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_mx(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t sfa, uint32_t sfb,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(MX_IDESC), "r"(accumulate), "r"(sfa), "r"(sfb));
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(taddr),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// 1-D bulk copy global -> shared completing on an mbarrier (no multicast)
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(mbar)
               : "memory");
}

// per-stage scale staging in shared memory: 128 A row scales + an 8-block window of B block scales
constexpr int SC_BYTES = 128 * 4 + 8 * 4;

// UE8M0 byte of a power-of-two fp32 scale (its biased exponent), in all four bytes
__device__ __forceinline__ uint32_t e8m0_word(float s) { return ((__float_as_uint(s) >> 23) & 0xffu) * 0x01010101u; }

__global__ void __launch_bounds__(320, 1)
gemm_mx_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
               const float* __restrict__ sa_t, const float* __restrict__ sb_t, __nv_bfloat16* __restrict__ C,
               float* __restrict__ C32, int M, int N, int K, int splits, int kper, int Mp, int NBp) {
  // sa_t [K/128, Mp] and sb_t [K/128, NBp]: scales MN-major, so the 128 row scales
  // of a tile's K block are one contiguous 512-byte run the TMA unit fetches with
  // the operand tiles
  constexpr int A_BYTES = BM * KB;
  constexpr int B_BYTES = MX_BN * KB;
  constexpr int ST = MX_STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = tc::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = base + ST * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + ST * (A_BYTES + B_BYTES));
  const uint32_t bar_full = tc::smem_u32(bars);
  const uint32_t bar_empty = bar_full + 8 * ST;
  const uint32_t bar_sfull = bar_empty + 8 * ST;
  const uint32_t bar_tfull = bar_sfull + 8 * ST;
  const uint32_t bar_tempty = bar_tfull + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * ST + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* sc_base = gbase + ST * (A_BYTES + B_BYTES) + 256;
  const uint32_t sSC = tc::smem_u32(sc_base);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + BM - 1) / BM, num_n = (N + MX_BN - 1) / MX_BN;
  const int num_kb = K / KB;
  const int num_units = num_m * num_n * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      tc::mbar_init(bar_full + 8 * s, 1);
      tc::mbar_init(bar_empty + 8 * s, 1);
      tc::mbar_init(bar_sfull + 8 * s, 4);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(bar_tfull + 8 * a, 1);
      tc::mbar_init(bar_tempty + 8 * a, 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tc::smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok && !*abort_flag; u += gridDim.x) {
        int mt, nt, kb0, kb1;
        unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % ST;
          const uint32_t ph = (it / ST) & 1;
          if (!wait(bar_empty + 8 * s, ph ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          tc::mbar_expect_tx(bar_full + 8 * s, A_BYTES + B_BYTES + SC_BYTES);
          tc::tma_load_2d(sA + s * A_BYTES, &tmap_a, bar_full + 8 * s, kb * KB, mt * BM);
          tc::tma_load_2d(sB + s * B_BYTES, &tmap_b, bar_full + 8 * s, kb * KB, nt * MX_BN);
          const int ws = ((nt * MX_BN) >> 7) & ~3;  // 16-byte aligned window of the tile's B blocks
          bulk_load(sSC + s * SC_BYTES, sa_t + (long long)kb * Mp + mt * BM, 512, bar_full + 8 * s);
          bulk_load(sSC + s * SC_BYTES + 512, sb_t + (long long)kb * NBp + ws, 32, bar_full + 8 * s);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int it = 0, local = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok && !*abort_flag; u += gridDim.x, ++local) {
        int mt, nt, kb0, kb1;
        unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
        const int acc = local & 1;
        if (!wait(bar_tempty + 8 * acc, ((local >> 1) & 1) ^ 1, abort_flag)) break;
        tc::tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * MX_BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % ST;
          const uint32_t ph = (it / ST) & 1;
          if (!wait(bar_full + 8 * s, ph, abort_flag) || !wait(bar_sfull + 8 * s, ph, abort_flag)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a0 = sA + s * A_BYTES, b0 = sB + s * B_BYTES;
          const uint32_t sfa = tmem_base + MX_SF_COL + s * 16, sfb = sfa + 8;
#pragma unroll
          for (int k = 0; k < KB / 32; ++k)
            umma_mx(tmem_d, tc::desc_kmajor_sw128(a0 + k * 32), tc::desc_kmajor_sw128(b0 + k * 32), sfa, sfb,
                    (kb > kb0 || k > 0) ? 1u : 0u);
          tc::umma_commit(bar_empty + 8 * s);
        }
        if (!ok) break;
        tc::umma_commit(bar_tfull + 8 * acc);
      }
    }
    __syncwarp();
  } else if (warp >= 6) {
    // scale writers: quadrant q = warp % 4 owns lanes 32q..32q+31 of every scale column
    const int quad = warp & 3;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      int mt, nt, kb0, kb1;
      unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
      const int ws = ((nt * MX_BN) >> 7) & ~3;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % ST;
        const uint32_t ph = (it / ST) & 1;
        // the stage's scales landed with its operand tiles; the stage (and so this
        // scale slot) was refilled only after the MMAs of stage it - ST completed
        if (!wait(bar_full + 8 * s, ph, abort_flag)) {
          ok = false;
          break;
        }
        const float* sc = reinterpret_cast<const float*>(sc_base + s * SC_BYTES);
        uint32_t wa[4], wb[8];
#pragma unroll
        for (int c = 0; c < 4; ++c) wa[c] = e8m0_word(sc[c * 32 + lane]);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int n = nt * MX_BN + c * 32 + lane;
          wb[c] = (c < MX_BN / 32 && n < N) ? e8m0_word(sc[128 + (n >> 7) - ws]) : 0x7f7f7f7fu;
        }
        tc::tc_fence_after();
        const uint32_t slot = tmem_base + lane_off + MX_SF_COL + s * 16;
        tmem_st4(slot, wa);
        tmem_st8(slot + 8, wb);
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_sfull + 8 * s);
      }
    }
  } else {
    // epilogue warps 2..5
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int local = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
      int mt, nt, kb0, kb1;
      unit_coords(u, num_m, num_n, splits, kper, num_kb, mt, nt, kb0, kb1);
      const int acc = local & 1;
      if (!wait(bar_tfull + 8 * acc, (local >> 1) & 1, abort_flag)) break;
      tc::tc_fence_after();
      const int m = mt * BM + row_in_tile;
      const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * MX_BN;
#pragma unroll 1
      for (int c = 0; c < MX_BN / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(trow + c * 32, r);
        const int n0 = nt * MX_BN + c * 32;
        if (m >= M || n0 >= N) continue;
        if (splits == 1) {
          __nv_bfloat16* dst = C + (long long)m * N + n0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (n0 + q * 8 < N) {
              uint4 v;
              uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[q * 8 + 2 * e]),
                                                         __uint_as_float(r[q * 8 + 2 * e + 1]));
                pv[e] = *reinterpret_cast<uint32_t*>(&h);
              }
              *reinterpret_cast<uint4*>(dst + q * 8) = v;
            }
          }
        } else {
          float* dst = C32 + (long long)m * N + n0;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (n0 + e < N) atomicAdd(dst + e, __uint_as_float(r[e]));
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_tempty + 8 * acc);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(512));
  }
}

// 2-D row-major byte tensor map, (box_rows x 128)-byte box, 128-byte swizzle.
inline CUtensorMap make_tmap_u8(const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "rl_b200: cuTensorMapEncodeTiled (u8) failed (", (int)r, ")");
  return m;
}

}  // namespace f8
}  // namespace rlb

using namespace rlb;

// a [M, K] e4m3, a_scale [M, K/128] fp32; b [N, K] e4m3, b_scale [ceil(N/128), K/128]
// fp32; returns bf16 [M, N].  splits = 0 picks a K split that fills the SMs
// when the output has fewer 128 x 128 tiles than SMs.
at::Tensor gemm_fp8(at::Tensor a, at::Tensor a_scale, at::Tensor b, at::Tensor b_scale, int64_t splits) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kFloat8_e4m3fn &&
                  b.scalar_type() == at::kFloat8_e4m3fn,
              "rl_b200 gemm_fp8: e4m3 CUDA operands expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.is_contiguous() && b.is_contiguous(),
              "rl_b200 gemm_fp8: contiguous a [M, K], b [N, K]");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(K % 128 == 0 && K > 0 && N % 8 == 0, "rl_b200 gemm_fp8: K % 128 == 0 and N % 8 == 0 required");
  const int num_kb = K / 128;
  TORCH_CHECK(a_scale.scalar_type() == at::kFloat && a_scale.is_contiguous() && a_scale.numel() == (int64_t)M * num_kb,
              "rl_b200 gemm_fp8: a_scale fp32 [M, K/128]");
  TORCH_CHECK(b_scale.scalar_type() == at::kFloat && b_scale.is_contiguous() &&
                  b_scale.numel() == (int64_t)((N + 127) / 128) * num_kb,
              "rl_b200 gemm_fp8: b_scale fp32 [ceil(N/128), K/128]");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "rl_b200 gemm_fp8: 16-byte aligned operands");
  const c10::cuda::CUDAGuard guard(a.device());
  auto c = at::empty({M, N}, a.options().dtype(at::kBFloat16));
  if (M == 0 || N == 0) return c;
  const int tiles = ((M + tc::BM - 1) / tc::BM) * ((N + f8::BN - 1) / f8::BN);
  int sp = (int)splits;
  if (sp <= 0) sp = tiles >= num_sms() ? 1 : std::max(1, num_sms() / tiles);
  sp = std::min(sp, num_kb);
  const int kper = (num_kb + sp - 1) / sp;
  sp = (num_kb + kper - 1) / kper;  // every split owns at least one K block
  at::Tensor c32;
  if (sp > 1) c32 = at::zeros({M, N}, a.options().dtype(at::kFloat));
  const CUtensorMap ta = f8::make_tmap_u8(a.data_ptr(), M, K, tc::BM);
  const CUtensorMap tb = f8::make_tmap_u8(b.data_ptr(), N, K, f8::BN);
  constexpr int STAGES = 6;
  const int smem = STAGES * (tc::BM * f8::KB + f8::BN * f8::KB) + 1024 + 256;
  auto kern = f8::gemm_f8_kernel<STAGES>;
  static bool attr_set = false;  // once: the call may run inside a CUDA-graph capture
  if (!attr_set) {
    RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  const int grid = std::min(tiles * sp, num_sms());
  kern<<<grid, f8::THREADS, smem, stream()>>>(ta, tb, a_scale.data_ptr<float>(), b_scale.data_ptr<float>(),
                                              (__nv_bfloat16*)c.data_ptr(), sp > 1 ? c32.data_ptr<float>() : nullptr,
                                              M, N, K, sp, kper);
  RLB_CUDA_CHECK(cudaGetLastError());
  if (sp > 1) c.copy_(c32);
  return c;
}

// Same product with power-of-two scales applied by the tensor cores (see
// gemm_mx_kernel).  Scales are MN-major: a_scale_t [K/128, Mp] (Mp >= M rounded
// up to 128; rl_b200._C.quant_fp8_group_t writes this layout) and b_scale_t
// [K/128, NBp] (NBp >= ceil(N/128) rounded up to 4, plus 4).  They must be exact
// powers of two (quantisers with pow2 = true); only their exponents are used.
at::Tensor gemm_mxf8(at::Tensor a, at::Tensor a_scale_t, at::Tensor b, at::Tensor b_scale_t, int64_t splits) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kFloat8_e4m3fn &&
                  b.scalar_type() == at::kFloat8_e4m3fn,
              "rl_b200 gemm_mxf8: e4m3 CUDA operands expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.is_contiguous() && b.is_contiguous(),
              "rl_b200 gemm_mxf8: contiguous a [M, K], b [N, K]");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(K % 128 == 0 && K > 0 && N % 8 == 0, "rl_b200 gemm_mxf8: K % 128 == 0 and N % 8 == 0 required");
  const int num_kb = K / 128;
  const int NB = (N + 127) / 128;
  TORCH_CHECK(a_scale_t.scalar_type() == at::kFloat && a_scale_t.is_contiguous() && a_scale_t.dim() == 2 &&
                  a_scale_t.size(0) == num_kb && a_scale_t.size(1) >= ((M + 127) / 128) * 128 &&
                  a_scale_t.size(1) % 128 == 0,
              "rl_b200 gemm_mxf8: a_scale_t fp32 [K/128, Mp], Mp a multiple of 128 covering M");
  TORCH_CHECK(b_scale_t.scalar_type() == at::kFloat && b_scale_t.is_contiguous() && b_scale_t.dim() == 2 &&
                  b_scale_t.size(0) == num_kb && b_scale_t.size(1) >= ((NB + 3) & ~3) + 4 && b_scale_t.size(1) % 4 == 0,
              "rl_b200 gemm_mxf8: b_scale_t fp32 [K/128, NBp], NBp % 4 == 0 and >= ceil(N/128) rounded to 4, + 4");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(a_scale_t.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(b_scale_t.data_ptr()) % 16 == 0,
              "rl_b200 gemm_mxf8: 16-byte aligned operands and scales");
  const c10::cuda::CUDAGuard guard(a.device());
  auto c = at::empty({M, N}, a.options().dtype(at::kBFloat16));
  if (M == 0 || N == 0) return c;
  const int tiles = ((M + tc::BM - 1) / tc::BM) * ((N + f8::MX_BN - 1) / f8::MX_BN);
  int sp = (int)splits;
  if (sp <= 0) sp = tiles >= num_sms() ? 1 : std::max(1, num_sms() / tiles);
  sp = std::min(sp, num_kb);
  const int kper = (num_kb + sp - 1) / sp;
  sp = (num_kb + kper - 1) / kper;
  at::Tensor c32;
  if (sp > 1) c32 = at::zeros({M, N}, a.options().dtype(at::kFloat));
  const CUtensorMap ta = f8::make_tmap_u8(a.data_ptr(), M, K, tc::BM);
  const CUtensorMap tb = f8::make_tmap_u8(b.data_ptr(), N, K, f8::MX_BN);
  const int smem = f8::MX_STAGES * (tc::BM * f8::KB + f8::MX_BN * f8::KB) + 1024 + 256 +
                   f8::MX_STAGES * f8::SC_BYTES;
  static bool attr_set = false;  // once: the call may run inside a CUDA-graph capture
  if (!attr_set) {
    RLB_CUDA_CHECK(cudaFuncSetAttribute(f8::gemm_mx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set = true;
  }
  const int grid = std::min(tiles * sp, num_sms());
  f8::gemm_mx_kernel<<<grid, 320, smem, stream()>>>(ta, tb, a_scale_t.data_ptr<float>(), b_scale_t.data_ptr<float>(),
                                                    (__nv_bfloat16*)c.data_ptr(),
                                                    sp > 1 ? c32.data_ptr<float>() : nullptr, M, N, K, sp, kper,
                                                    (int)a_scale_t.size(1), (int)b_scale_t.size(1));
  RLB_CUDA_CHECK(cudaGetLastError());
  if (sp > 1) c.copy_(c32);
  return c;
}

int64_t gemm_fp8_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, f8::g_f8_error, sizeof(int)));
  if (reset) {
    int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(f8::g_f8_error, &z, sizeof(int)));
  }
  return v;
}
