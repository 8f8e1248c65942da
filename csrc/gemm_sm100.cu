// General bf16 GEMM on the 5th-generation tensor cores (sm_100a): every product
// of a linear layer's forward and backward pass.
//
//   C[M, N] = op(A) x op(B)^T      (fp32 accumulation in tensor memory)
//
// Operand majors (both row-major in memory):
//   A K-major  : A stored [M, K]          A MN-major : A stored [K, M]
//   B K-major  : B stored [N, K]          B MN-major : B stored [K, N]
// so a linear layer y = x W^T (W [N, K]) uses
//   forward  y  = x  W^T : A = x  [T, K] K-major,  B = W  [N, K] K-major
//   dgrad    dx = dy W   : A = dy [T, N] K-major,  B = W  [N, K] MN-major (reduce over N)
//   wgrad    dW = dy^T x : A = dy [T, N] MN-major, B = x  [T, K] MN-major (reduce over T)
// Epilogues: bf16 store, fp32 store, or fp32 read-add-write (the weight gradient
// accumulated straight into an fp32 main-grad buffer; each output tile has one
// owner, so no atomics).  Two more serve the LM head of the RL losses, where the
// product is the logits of a vocabulary (shard) and must never reach HBM:
//   EPI_LOGPROB : each epilogue thread owns one token row of the tile and reduces
//                 its 256 logits (scaled by 1/temperature) to the online-softmax
//                 state (max, sum exp, sum x exp) of that tile, written as
//                 [3, num_n_tiles, M] fp32 partials, plus the target's logit; a
//                 small kernel then merges the partials over the tiles.
//   EPI_DLOGITS : the backward recomputes the tile and stores
//                 dlogits = dlogp / T * (onehot(target) - exp(x / T - lse)) in bf16,
//                 the input of the dgrad / wgrad products (no logits pass between).
//
// Two tile shapes, one source:
//   PAIR = false : one CTA per SM computes 128 x 256 tiles (tcgen05.mma.cta_group::1,
//                  M = 128, N = 256); stage = A 128x64 + B 256x64 (48 KB), 4 stages.
//   PAIR = true  : a 2-CTA cluster computes 256 x 256 tiles with
//                  tcgen05.mma.cta_group::2 (M = 256, N = 256) issued by the
//                  even CTA: each CTA stages ITS OWN half of A (128 rows) and of B
//                  (128 output columns) in its own shared memory, so per MMA FLOP a
//                  CTA loads a third less than in the 1-CTA tile (the B operand is
//                  split between the pair instead of re-read by both).  Stage =
//                  32 KB per CTA, 6 stages.  Every TMA load is a plain one: it reads
//                  this GPU's memory into the loading CTA's own shared memory; the
//                  odd CTA's loads signal the even CTA's mbarrier (.cta_group::2).
//
// Roles (6 warps): warp 0 = TMA producer (one lane), warp 1 = tensor-memory
// allocator and MMA issuer (one lane; in a pair only the even CTA issues),
// warps 2-5 = epilogue (tcgen05.ld of the warp's TMEM lane quadrant).  Two
// 256-column fp32 accumulators (all 512 TMEM columns) let the epilogue of tile
// i overlap the MMAs of tile i + 1.  Persistent: tiles are visited in a grouped
// raster (8 row-tiles per column sweep) for L2 reuse.
//
// Every mbarrier wait is bounded: on expiry the kernel records an error code in
// g_gemm_error (read from the host by gemm_sm100_error_flag), raises a CTA-wide
// abort flag so all roles leave their loops, waits (bounded) for its loads in
// flight, frees tensor memory and returns.
//
// Swizzle / descriptor facts used here (PTX ISA, tcgen05 shared-memory
// descriptor; CUTLASS's canonical SW128 layouts):
//   K-major  tile: rows of 64 elements (128 B), 8-row groups 1024 B apart
//                  (SBO = 1024); a K-step of 16 advances the start by 32 B.
//   MN-major tile: TMA boxes of 64 (MN, contiguous) x 64 (K rows), 8 KB each,
//                  placed one after another along MN: LBO = 8192 B (next 64-wide
//                  MN atom), SBO = 1024 B (next 8 K-rows); a K-step of 16
//                  advances the start by 16 rows = 2048 B.
#include "tc_common.cuh"

namespace rlb {
namespace g100 {

using namespace rlb::tc;

__device__ int g_gemm_error = 0;

constexpr int EPI_BF16 = 0;     // C bf16 = acc
constexpr int EPI_F32 = 1;      // C fp32 = acc
constexpr int EPI_F32_ADD = 2;  // C fp32 += acc
constexpr int EPI_LOGPROB = 3;  // per-tile softmax partials of acc / T (C unused)
constexpr int EPI_DLOGITS = 4;  // C bf16 = d logprob / d logits
constexpr int GROUP = 8;

// Per-row inputs / outputs of the two LM-head epilogues (unused otherwise).
struct LpArgs {
  const long long* tgt;  // [M] target id within this vocabulary shard (outside [0, N): not in this shard)
  const float* lse;      // [M] log-sum-exp of the whole (all-shard) row       (EPI_DLOGITS)
  const float* dlp;      // [M] d loss / d logprob                             (EPI_DLOGITS)
  float* part;           // [3, num_n, M] tile max, sum exp, sum x*exp         (EPI_LOGPROB)
  float* xt;             // [M] target logit / T; pre-zeroed                  (EPI_LOGPROB)
  float inv_temp;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// Arrive (with expected transaction bytes) on a barrier named by its cluster
// address.  Default (CTA-scope) semantics: the data these barriers guard moves
// through the async proxy (TMA writes, MMA reads, TMEM loads fenced with
// tcgen05.fence), whose completion the barrier mechanism itself orders; a
// cluster-scope release here would put a cluster-wide memory barrier on the
// producer's and the epilogue's critical path for nothing.
__device__ __forceinline__ void mbar_expect_tx_cl(uint32_t caddr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;\n" ::"r"(caddr), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cl(uint32_t caddr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" ::"r"(caddr) : "memory");
}
__device__ __forceinline__ bool mbar_test_cl(uint32_t addr, uint32_t parity) { return mbar_test(addr, parity); }
// Bounded wait on a barrier of this CTA (its arrivals may come from the peer CTA).
__device__ __forceinline__ bool wait_bar(uint32_t addr, uint32_t parity, volatile int* abort_flag, int code) {
  const long long t0 = clock64();
  while (!mbar_test_cl(addr, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicExch(&g_gemm_error, code);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// 2-D tile load into this CTA's shared memory; completion bytes go to `mbar`,
// a barrier of this CTA (PAIR = false) or of the pair's even CTA (PAIR = true).
template <bool PAIR>
__device__ __forceinline__ void tma_2d(uint32_t dst, const void* tmap, uint32_t mbar, int x, int y) {
  if constexpr (PAIR) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
        "l"(tmap), "r"(mbar), "r"(x), "r"(y)
        : "memory");
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];\n" ::"r"(dst),
        "l"(tmap), "r"(mbar), "r"(x), "r"(y)
        : "memory");
  }
}

template <bool PAIR>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  if constexpr (PAIR) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  }
}

// Arrive on `bar` once every MMA issued so far completed; in a pair the arrive
// goes to the barrier at the same offset in both CTAs: one commit to this CTA's
// barrier and one to the peer's (its address in the cluster window).
template <bool PAIR>
__device__ __forceinline__ void commit(uint32_t bar) {
  if constexpr (PAIR) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mapa(bar, 1))
                 : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
  }
}

// Shared-memory descriptor of an MN-major SW128 tile (see the header comment).
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(8192u >> 4) << 16;  // LBO: next 64-element MN atom
  d |= (uint64_t)(1024u >> 4) << 32;  // SBO: next 8 K-rows
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__device__ __forceinline__ void tile_of(int tile, int num_m, int num_n, int& mt, int& nt) {
  const int group = GROUP * num_n;
  const int gid = tile / group;
  const int first_m = gid * GROUP;
  const int gsize = min(num_m - first_m, GROUP);
  const int in = tile % group;
  mt = first_m + in % gsize;
  nt = in / gsize;
}

template <bool PAIR, bool A_MN, bool B_MN>
struct Cfg {
  static constexpr int TM = PAIR ? 256 : 128;  // output rows per tile (MMA M)
  static constexpr int TN = 256;               // output columns per tile (MMA N)
  static constexpr int CM = 128;               // A rows staged by one CTA
  static constexpr int CN = PAIR ? 128 : 256;  // B rows (output columns) staged by one CTA
  static constexpr int A_BYTES = CM * BK * 2;
  static constexpr int B_BYTES = CN * BK * 2;
  static constexpr int STAGES = PAIR ? 6 : 4;
  static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + 1024 + 256;
  static constexpr uint32_t IDESC =
      idesc_bf16(TM, TN) | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16);
};

template <bool PAIR, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1)
gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, void* __restrict__ C,
            int M, int N, int K, long long ldc, const LpArgs lp) {
  using G = Cfg<PAIR, A_MN, B_MN>;
  constexpr int STAGES = G::STAGES;
  constexpr int A_BYTES = G::A_BYTES, B_BYTES = G::B_BYTES;
  constexpr uint32_t TMEM_COLS = 512;
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
  const uint32_t crank = PAIR ? cluster_rank() : 0u;
  const bool leader = crank == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // pair (or CTA) index
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int num_m = (M + G::TM - 1) / G::TM, num_n = (N + G::TN - 1) / G::TN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, PAIR ? 2 : 1);  // one expect-tx arrive per loading CTA
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull + 8 * a, 1);
      mbar_init(bar_tempty + 8 * a, PAIR ? 8 : 4);  // every epilogue warp of the pair
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::);
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the barriers every role signals: the pair's even CTA owns "full" and "tmem empty"
  const uint32_t full_dst = PAIR ? mapa(bar_full, 0) : bar_full;
  const uint32_t tempty_dst = PAIR ? mapa(bar_tempty, 0) : bar_tempty;

  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      for (int tile = unit; tile < num_tiles && !*abort_flag; tile += units) {
        int mt, nt;
        tile_of(tile, num_m, num_n, mt, nt);
        const int a_row = mt * G::TM + (int)crank * G::CM;  // this CTA's A rows
        const int b_row = nt * G::TN + (int)crank * G::CN;  // this CTA's output columns
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_bar(bar_empty + 8 * s, ph ^ 1, abort_flag, 1)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_dst + 8 * s;
          if constexpr (PAIR) mbar_expect_tx_cl(fb, A_BYTES + B_BYTES);
          else mbar_expect_tx(fb, A_BYTES + B_BYTES);
          const uint32_t da = sA + s * A_BYTES, db = sB + s * B_BYTES;
          if constexpr (A_MN) {
#pragma unroll
            for (int j = 0; j < G::CM / 64; ++j) tma_2d<PAIR>(da + j * 8192, &tmap_a, fb, a_row + 64 * j, kb * BK);
          } else {
            tma_2d<PAIR>(da, &tmap_a, fb, kb * BK, a_row);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < G::CN / 64; ++j) tma_2d<PAIR>(db + j * 8192, &tmap_b, fb, b_row + 64 * j, kb * BK);
          } else {
            tma_2d<PAIR>(db, &tmap_b, fb, kb * BK, b_row);
          }
        }
        if (!ok) break;
      }
      // error path: before leaving, let this CTA's loads in flight land (bounded); a
      // pair's loads all count on the even CTA's barriers
      if (*abort_flag && leader) {
        for (int j = max(0, it - STAGES); j < it; ++j) {
          const long long t0 = clock64();
          while (!mbar_test_cl(bar_full + 8 * (j % STAGES), (j / STAGES) & 1) && clock64() - t0 < kWaitCycles) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int it = 0, local = 0;
      for (int tile = unit; tile < num_tiles && !*abort_flag; tile += units, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!wait_bar(bar_tempty + 8 * acc, aph ^ 1, abort_flag, 2)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * G::TN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_bar(bar_full + 8 * s, ph, abort_flag, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = sA + s * A_BYTES, b0 = sB + s * B_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? desc_mn_sw128(a0 + k * 2048) : desc_kmajor_sw128(a0 + k * 32);
            const uint64_t bd = B_MN ? desc_mn_sw128(b0 + k * 2048) : desc_kmajor_sw128(b0 + k * 32);
            mma<PAIR>(tmem_d, ad, bd, G::IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          commit<PAIR>(bar_empty + 8 * s);
        }
        if (!ok) break;
        commit<PAIR>(bar_tfull + 8 * acc);
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5: TMEM lane quadrant = warp % 4 (rows quad*32 .. +31 of this CTA's half)
    const int quad = warp & 3;
    const int row_in = (int)crank * 128 + quad * 32 + lane;
    int local = 0;
    for (int tile = unit; tile < num_tiles; tile += units, ++local) {
      int mt, nt;
      tile_of(tile, num_m, num_n, mt, nt);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!wait_bar(bar_tfull + 8 * acc, aph, abort_flag, 4)) break;
      tc_fence_after();
      const int m = mt * G::TM + row_in;
      const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * G::TN;
      // LM-head epilogues: this thread's row state
      [[maybe_unused]] long long tgt = -1;
      [[maybe_unused]] float lm = -INFINITY, ls = 0.f, lu = 0.f, gsc = 0.f, lrow = 0.f;
      if constexpr (EPI == EPI_LOGPROB || EPI == EPI_DLOGITS) {
        if (m < M) tgt = lp.tgt[m];
        if constexpr (EPI == EPI_DLOGITS) {
          if (m < M) {
            gsc = lp.dlp[m] * lp.inv_temp;
            lrow = lp.lse[m];
          }
        }
      }
#pragma unroll 1
      for (int c = 0; c < G::TN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + c * 32, r);
        const int n0 = nt * G::TN + c * 32;
        if (m >= M || n0 >= N) continue;
        const bool full = n0 + 32 <= N;
        if constexpr (EPI == EPI_LOGPROB) {
          float f[32];
          float cm = -INFINITY;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            f[j] = (full || n0 + j < N) ? __uint_as_float(r[j]) * lp.inv_temp : -INFINITY;
            cm = fmaxf(cm, f[j]);
          }
          if (cm > lm) {  // one rescale per 32 columns
            const float sc = __expf(lm - cm);
            ls *= sc;
            lu *= sc;
            lm = cm;
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float e = __expf(f[j] - lm);
            ls += e;
            lu += e > 0.f ? f[j] * e : 0.f;  // masked columns: e = 0 (and f = -inf)
          }
          const long long d = tgt - n0;
          if (d >= 0 && d < 32 && tgt < N) {  // a target past the shard's edge belongs to another shard
            float xv = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) xv = (j == (int)d) ? f[j] : xv;
            lp.xt[m] = xv;
          }
        } else if constexpr (EPI == EPI_DLOGITS) {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (long long)m * ldc + n0;
          float g[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float p = __expf(__uint_as_float(r[j]) * lp.inv_temp - lrow);
            g[j] = gsc * ((tgt == (long long)(n0 + j) ? 1.f : 0.f) - p);
          }
          if (full && (ldc % 8) == 0) {
            uint4 v[4];
            uint32_t* pv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              __nv_bfloat162 h = __floats2bfloat162_rn(g[2 * j], g[2 * j + 1]);
              pv[j] = *reinterpret_cast<uint32_t*>(&h);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = v[j];
          } else {
            for (int j = 0; j < 32; ++j)
              if (n0 + j < N) dst[j] = __float2bfloat16_rn(g[j]);
          }
        } else if constexpr (EPI == EPI_BF16) {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (long long)m * ldc + n0;
          if (full && (ldc % 8) == 0) {
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
            for (int j = 0; j < 32; ++j)
              if (n0 + j < N) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        } else {
          float* dst = reinterpret_cast<float*>(C) + (long long)m * ldc + n0;
          if (full && (ldc % 4) == 0) {
            float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                     __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
              if constexpr (EPI == EPI_F32_ADD) {
                const float4 o = d4[j];
                v.x += o.x;
                v.y += o.y;
                v.z += o.z;
                v.w += o.w;
              }
              d4[j] = v;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (n0 + j < N) {
                const float v = __uint_as_float(r[j]);
                dst[j] = (EPI == EPI_F32_ADD) ? dst[j] + v : v;
              }
          }
        }
      }
      if constexpr (EPI == EPI_LOGPROB) {
        if (m < M) {
          const long long plane = (long long)num_n * M;
          const long long o = (long long)nt * M + m;
          lp.part[o] = lm;
          lp.part[plane + o] = ls;
          lp.part[2 * plane + o] = lu;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cl(tempty_dst + 8 * acc);
        else mbar_arrive(bar_tempty + 8 * acc);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) {
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
    } else {
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
    }
  }
}

// Merge the per-tile softmax states of EPI_LOGPROB over the vocabulary tiles:
// part [3, nt, M] -> m, s, u [M].  Block = 32 rows x 8 warps; warp w merges tiles
// w, w + 8, ... of its lane's row (loads coalesced over 32 consecutive rows), then
// the 8 warp states are merged through shared memory.
__global__ void __launch_bounds__(256)
lp_tile_merge_kernel(const float* __restrict__ part, int nt, int M, float* __restrict__ m_out,
                     float* __restrict__ s_out, float* __restrict__ u_out) {
  __shared__ float sh[3][8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int row = blockIdx.x * 32 + lane;
  const long long plane = (long long)nt * M;
  float m = -INFINITY, s = 0.f, u = 0.f;
  if (row < M) {
    for (int t = w; t < nt; t += 8) {
      const long long o = (long long)t * M + row;
      const float tm = part[o], ts = part[plane + o], tu = part[2 * plane + o];
      if (tm == -INFINITY) continue;
      if (tm > m) {
        const float f = __expf(m - tm);  // m = -inf -> 0
        s = s * f + ts;
        u = u * f + tu;
        m = tm;
      } else {
        const float f = __expf(tm - m);
        s += ts * f;
        u += tu * f;
      }
    }
  }
  sh[0][w][lane] = m;
  sh[1][w][lane] = s;
  sh[2][w][lane] = u;
  __syncthreads();
  if (w == 0 && row < M) {
    float M_ = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) M_ = fmaxf(M_, sh[0][i][lane]);
    float S = 0.f, U = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float tm = sh[0][i][lane];
      if (tm == -INFINITY) continue;
      const float f = __expf(tm - M_);
      S += sh[1][i][lane] * f;
      U += sh[2][i][lane] * f;
    }
    m_out[row] = M_;
    s_out[row] = S;
    u_out[row] = U;
  }
}

}  // namespace g100
}  // namespace rlb

using namespace rlb;

namespace {

// Row-major [rows, cols] bf16 matrix as a 2-D tensor map with a (box_cols x box_rows)
// box, 128-byte swizzle; out-of-bounds elements read as zero.
CUtensorMap tmap_bf16(const void* ptr, int64_t rows, int64_t cols, int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "rl_b200 gemm_sm100: cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

template <bool PAIR, bool A_MN, bool B_MN, int EPI>
void launch(const at::Tensor& a, const at::Tensor& b, void* c, int M, int N, int K, long long ldc, int max_units,
            const g100::LpArgs& lp = g100::LpArgs{}) {
  using G = g100::Cfg<PAIR, A_MN, B_MN>;
  // K-major operands: box = 64 K-columns x staged rows; MN-major: 64 x 64 boxes
  const CUtensorMap ta = A_MN ? tmap_bf16(a.data_ptr(), K, M, 64, 64) : tmap_bf16(a.data_ptr(), M, K, 64, G::CM);
  const CUtensorMap tb = B_MN ? tmap_bf16(b.data_ptr(), K, N, 64, 64) : tmap_bf16(b.data_ptr(), N, K, 64, G::CN);
  auto kern = g100::gemm_kernel<PAIR, A_MN, B_MN, EPI>;
  RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
  const int tiles = ((M + G::TM - 1) / G::TM) * ((N + G::TN - 1) / G::TN);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = G::SMEM;
  cfg.stream = stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = PAIR ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // A persistent grid must be resident all at once: a CTA pair needs two free SMs of
  // one GPC, and GPCs with an odd SM count leave one SM without a partner, so the
  // number of co-resident pairs is below SMs / 2.  Ask the occupancy calculator
  // (once per device and variant) instead of assuming it.
  static int resident[64] = {0};
  int dev = 0;
  RLB_CUDA_CHECK(cudaGetDevice(&dev));
  int& res = resident[dev & 63];
  if (res == 0) {
    cfg.gridDim = dim3(2 * (PAIR ? 2 : 1));
    int n = 0;
    RLB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    res = std::max(1, n);
  }
  const int units = std::max(1, std::min({tiles, max_units, res}));
  cfg.gridDim = dim3(units * (PAIR ? 2 : 1));
  RLB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, c, M, N, K, ldc, lp));
}

template <bool PAIR, int EPI>
void dispatch_major(bool a_mn, bool b_mn, const at::Tensor& a, const at::Tensor& b, void* c, int M, int N, int K,
                    long long ldc, int max_units) {
  if (!a_mn && !b_mn) launch<PAIR, false, false, EPI>(a, b, c, M, N, K, ldc, max_units);
  else if (!a_mn && b_mn) launch<PAIR, false, true, EPI>(a, b, c, M, N, K, ldc, max_units);
  else if (a_mn && !b_mn) launch<PAIR, true, false, EPI>(a, b, c, M, N, K, ldc, max_units);
  else launch<PAIR, true, true, EPI>(a, b, c, M, N, K, ldc, max_units);
}

}  // namespace

// out (M x N) = op(a) op(b)^T, see the header comment.
//   a: [M, K] (a_mn = false) or [K, M] (a_mn = true), bf16, contiguous
//   b: [N, K] (b_mn = false) or [K, N] (b_mn = true), bf16, contiguous
//   out: [M, N] contiguous; bf16 (accumulate must be false) or fp32 (out = or += the product)
//   tile: 0 = choose (2-CTA 256x256 when it fills the GPU), 1 = 1-CTA 128x256, 2 = 2-CTA 256x256
void gemm_sm100(at::Tensor a, at::Tensor b, at::Tensor out, bool a_mn, bool b_mn, bool accumulate, int64_t tile) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "rl_b200 gemm_sm100: CUDA tensors expected");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "rl_b200 gemm_sm100: bf16 operands expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "rl_b200 gemm_sm100: 2-D operands");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && out.is_contiguous(), "rl_b200 gemm_sm100: contiguous operands");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  const int Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb && K > 0, "rl_b200 gemm_sm100: reduction sizes differ");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "rl_b200 gemm_sm100: out must be [M, N]");
  TORCH_CHECK(a.size(1) % 8 == 0 && b.size(1) % 8 == 0,
              "rl_b200 gemm_sm100: the contiguous dimension of each operand must be a multiple of 8 (16-byte rows)");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "rl_b200 gemm_sm100: operands must be 16-byte aligned");
  const bool f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || (out.scalar_type() == at::kBFloat16 && !accumulate),
              "rl_b200 gemm_sm100: out is bf16 (overwrite) or fp32 (overwrite or accumulate)");
  if (M == 0 || N == 0) return;
  const c10::cuda::CUDAGuard guard(a.device());
  const int sms = num_sms();
  const long long t2 = (long long)((M + 255) / 256) * ((N + 255) / 256);
  const bool pair = tile == 2 || (tile == 0 && t2 >= sms / 2);
  void* c = out.data_ptr();
  const long long ldc = N;
  if (pair) {
    if (!f32) dispatch_major<true, g100::EPI_BF16>(a_mn, b_mn, a, b, c, M, N, K, ldc, sms / 2);
    else if (accumulate) dispatch_major<true, g100::EPI_F32_ADD>(a_mn, b_mn, a, b, c, M, N, K, ldc, sms / 2);
    else dispatch_major<true, g100::EPI_F32>(a_mn, b_mn, a, b, c, M, N, K, ldc, sms / 2);
  } else {
    if (!f32) dispatch_major<false, g100::EPI_BF16>(a_mn, b_mn, a, b, c, M, N, K, ldc, sms);
    else if (accumulate) dispatch_major<false, g100::EPI_F32_ADD>(a_mn, b_mn, a, b, c, M, N, K, ldc, sms);
    else dispatch_major<false, g100::EPI_F32>(a_mn, b_mn, a, b, c, M, N, K, ldc, sms);
  }
}

int64_t gemm_sm100_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g100::g_gemm_error, sizeof(int)));
  if (reset) {
    int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(g100::g_gemm_error, &z, sizeof(int)));
  }
  return v;
}

namespace {

void check_lm_head(const at::Tensor& h, const at::Tensor& w, const at::Tensor& targets) {
  TORCH_CHECK(h.is_cuda() && w.is_cuda() && targets.is_cuda(), "rl_b200 lm-head gemm: CUDA tensors expected");
  TORCH_CHECK(h.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16,
              "rl_b200 lm-head gemm: bf16 hidden states and weight expected");
  TORCH_CHECK(h.dim() == 2 && w.dim() == 2 && h.is_contiguous() && w.is_contiguous() && h.size(1) == w.size(1),
              "rl_b200 lm-head gemm: hidden [T, H] and weight [V, H], contiguous");
  TORCH_CHECK(h.size(1) % 8 == 0, "rl_b200 lm-head gemm: hidden size must be a multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
              "rl_b200 lm-head gemm: operands must be 16-byte aligned");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.dim() == 1 && targets.size(0) == h.size(0) &&
                  targets.is_contiguous(),
              "rl_b200 lm-head gemm: targets int64 [T]");
}

template <int EPI>
void launch_nt(const at::Tensor& a, const at::Tensor& b, void* c, int M, int N, int K, long long ldc,
               const g100::LpArgs& lp) {
  const int sms = num_sms();
  const long long t2 = (long long)((M + 255) / 256) * ((N + 255) / 256);
  if (t2 >= sms / 2) launch<true, false, false, EPI>(a, b, c, M, N, K, ldc, sms / 2, lp);
  else launch<false, false, false, EPI>(a, b, c, M, N, K, ldc, sms, lp);
}

}  // namespace

// LM head fused with the log-prob reductions (forward): for hidden [T, H] and this
// rank's vocabulary shard weight [V, H], returns per row (max, sum exp, sum x exp,
// target logit) of x = hidden @ weight^T / temperature over the shard, fp32 [T]
// each; targets are ids within the shard (others contribute no target logit).
// The logits exist only in tensor memory.
std::vector<at::Tensor> gemm_logprob_partials(at::Tensor h, at::Tensor w, at::Tensor targets, double temperature) {
  check_lm_head(h, w, targets);
  const c10::cuda::CUDAGuard guard(h.device());
  const int M = h.size(0), N = w.size(0), K = h.size(1);
  auto o = h.options().dtype(at::kFloat);
  auto m = at::empty({M}, o), s = at::empty({M}, o), u = at::empty({M}, o), xt = at::zeros({M}, o);
  if (M == 0 || N == 0) return {m.fill_(-INFINITY), s.zero_(), u.zero_(), xt};
  const int nt = (N + 255) / 256;
  auto part = at::empty({3, nt, M}, o);
  g100::LpArgs lp{};
  lp.tgt = reinterpret_cast<const long long*>(targets.data_ptr<int64_t>());
  lp.part = part.data_ptr<float>();
  lp.xt = xt.data_ptr<float>();
  lp.inv_temp = (float)(1.0 / temperature);
  launch_nt<g100::EPI_LOGPROB>(h, w, nullptr, M, N, K, N, lp);
  g100::lp_tile_merge_kernel<<<(M + 31) / 32, 256, 0, stream()>>>(part.data_ptr<float>(), nt, M, m.data_ptr<float>(),
                                                                  s.data_ptr<float>(), u.data_ptr<float>());
  RLB_CUDA_CHECK(cudaGetLastError());
  return {m, s, u, xt};
}

// LM head fused with the log-prob gradient (backward): recomputes the logits tile
// and writes dlogits = dlp / T * (onehot(target) - exp(x / T - lse)) as bf16 [T, V].
at::Tensor gemm_dlogits(at::Tensor h, at::Tensor w, at::Tensor targets, at::Tensor lse, at::Tensor dlp,
                        double temperature) {
  check_lm_head(h, w, targets);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && dlp.scalar_type() == at::kFloat && lse.is_contiguous() &&
                  dlp.is_contiguous() && lse.numel() == h.size(0) && dlp.numel() == h.size(0),
              "rl_b200 gemm_dlogits: lse and dlp fp32 [T]");
  const c10::cuda::CUDAGuard guard(h.device());
  const int M = h.size(0), N = w.size(0), K = h.size(1);
  auto out = at::empty({M, N}, h.options());
  if (M == 0 || N == 0) return out;
  g100::LpArgs lp{};
  lp.tgt = reinterpret_cast<const long long*>(targets.data_ptr<int64_t>());
  lp.lse = lse.data_ptr<float>();
  lp.dlp = dlp.data_ptr<float>();
  lp.inv_temp = (float)(1.0 / temperature);
  launch_nt<g100::EPI_DLOGITS>(h, w, out.data_ptr(), M, N, K, N, lp);
  return out;
}
