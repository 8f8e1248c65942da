// Flash-attention forward on the 5th-generation tensor cores (sm_100a), head
// dim 128, bf16, variable-length causal / full attention with grouped KV heads.
//
// One CTA computes one 128-query tile of one head (the q tiles of a sequence
// are visited longest-first for causal balance).  Per key block of 64 keys:
//
//   S_j = Q K_j^T        tcgen05.mma (M=128, N=64,  K=128), fp32 in TMEM
//   P_j = exp2(S_j*c - m) softmax warps: thread r owns query row r (TMEM lane r)
//   O  += P_j V_j        tcgen05.mma (M=128, N=128, K=64), fp32 in TMEM
//
// Operands: Q (K-major, 2 TMA boxes of 128 rows x 64 dims), K_j (K-major,
// 2 boxes of 64 keys x 64 dims), V_j read as the MN-major B operand (V is stored
// [keys, hd] with hd contiguous: 2 boxes of 64 dims x 64 keys, LBO = 8 KB to the
// next 64 dims, SBO = 1 KB to the next 8 keys).  P_j is written by the softmax
// warps as bf16 in the 128-byte-swizzled K-major layout straight into the
// shared-memory slot that held K_j (consumed by S_j, which completed before the
// softmax could read it), so the K/V ring needs no separate P buffer:
// smem = Q 32 KB + 2 stages x (K 16 KB + V 16 KB) = 96 KB, and two CTAs share an
// SM (one CTA's softmax overlaps the other's MMAs; TMEM 256 columns each).
//
// Within a CTA the MMA warp issues S_{j+1} (double-buffered in TMEM) before it
// waits for P_j, so QK^T of the next block overlaps the softmax of this one.
// The running max is updated lazily: the output is rescaled (tcgen05.ld/st of
// the O accumulator) only when a row's block max exceeds the max in use by more
// than 8 (log2 units); otherwise P is formed against the stale max (values at
// most 2^8, exact in the fp32 sums).  Queries beyond the sequence are computed
// and dropped; keys beyond it are masked, so TMA may read neighbouring
// sequences' rows (or zero-filled rows past the tensor end).
//
// Context parallelism: with cp_flags the producer waits, per key block, for the
// flag of the rank whose chunk holds the block (K/V still landing from peers).
//
// Every wait is bounded: on expiry g_attn_tc_error is set (read by
// attn_tc_error_flag), the roles leave their loops, tensor memory is freed.
#include "tc_common.cuh"

namespace rlb {
namespace fa {

using namespace rlb::tc;

__device__ int g_attn_tc_error = 0;

constexpr int HD = 128;
constexpr int BQ = 128;  // queries per CTA
constexpr int BKV = 64;  // keys per block
constexpr int Q_BYTES = BQ * HD * 2;    // 32 KB
constexpr int K_BYTES = BKV * HD * 2;   // 16 KB
constexpr int V_BYTES = BKV * HD * 2;   // 16 KB
constexpr int STAGES = 2;
constexpr int SMEM = Q_BYTES + STAGES * (K_BYTES + V_BYTES) + 1024 + 256;
constexpr uint32_t TMEM_COLS = 256;     // S double buffer (2 x 64) + O (128)
constexpr uint32_t IDESC_S = idesc_bf16(BQ, BKV);                    // Q K^T: both K-major
constexpr uint32_t IDESC_O = idesc_bf16(BQ, HD) | (1u << 16);         // P V: B (V) MN-major
constexpr float RESCALE_THRESHOLD = 8.0f;

__device__ __forceinline__ bool fwait(uint32_t addr, uint32_t parity, volatile int* abort_flag, int code) {
  return mbar_wait_err(addr, parity, abort_flag, &g_attn_tc_error, code);
}

__device__ __forceinline__ uint64_t desc_mn(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(8192u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__device__ __forceinline__ void tma_3d(uint32_t dst, const void* tmap, uint32_t mbar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];\n" ::"r"(
          dst),
      "l"(tmap), "r"(mbar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ bool cp_flag_ready(const uint32_t* p, uint32_t v) {
  uint32_t x;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(x) : "l"(p) : "memory");
  return (int)(x - v) >= 0;
}

__global__ void __launch_bounds__(192, 2)
fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const int* __restrict__ cu, int nq, int nkv, float scale_log2,
                 int causal, __nv_bfloat16* __restrict__ o, float* __restrict__ lse, int T_total,
                 const int* __restrict__ seg, const uint32_t* __restrict__ cp_flags, uint32_t cp_epoch, int cp_size,
                 long long wait_cycles) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base;
  const uint32_t sK = sQ + Q_BYTES;                 // stage s: sK + s * K_BYTES (P_j reuses it)
  const uint32_t sV = sK + STAGES * K_BYTES;        // stage s: sV + s * V_BYTES
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + Q_BYTES + STAGES * (K_BYTES + V_BYTES));
  const uint32_t bar_q = smem_u32(bars);
  const uint32_t bar_full = bar_q + 8;               // [STAGES]
  const uint32_t bar_empty = bar_full + 8 * STAGES;  // [STAGES]
  const uint32_t bar_s = bar_empty + 8 * STAGES;     // [2] S_j ready (MMA -> softmax)
  const uint32_t bar_sfree = bar_s + 16;             // [2] S buffer read (softmax -> MMA)
  const uint32_t bar_p = bar_sfree + 16;             // P_j written, O rescaled (softmax -> MMA)
  const uint32_t bar_o = bar_p + 8;                  // PV_j complete (MMA -> softmax)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 1 + 4 * STAGES + 2 + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int mblk = gridDim.y - 1 - blockIdx.y;
  const int b = blockIdx.z;
  const int s0 = seg ? seg[4 * b] : cu[b];
  const int L = seg ? seg[4 * b + 1] : cu[b + 1] - s0;
  const int k0 = seg ? seg[4 * b + 2] : s0;
  const int Lk = seg ? seg[4 * b + 3] : L;
  const int off = Lk - L;
  const int m0 = mblk * BQ;
  if (m0 >= L) return;
  const int kvh = h / (nq / nkv);
  const int n_end = causal ? min(Lk, m0 + BQ + off) : Lk;
  const int nblk = max(0, (n_end + BKV - 1) / BKV);

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_s + 8 * i, 1);
      mbar_init(bar_sfree + 8 * i, 4);
    }
    mbar_init(bar_p, 4);
    mbar_init(bar_o, 1);
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
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o = tmem + 2 * BKV;  // O accumulator columns [128, 256)

  if (warp == 0) {
    if (lane == 0 && nblk > 0) {
      mbar_expect_tx(bar_q, Q_BYTES);
      tma_3d(sQ, &tq, bar_q, 0, h, s0 + m0);
      tma_3d(sQ + Q_BYTES / 2, &tq, bar_q, 64, h, s0 + m0);
      for (int j = 0; j < nblk && !*abort_flag; ++j) {
        const int s = j % STAGES;
        if (!fwait(bar_empty + 8 * s, ((j / STAGES) & 1) ^ 1, abort_flag, 1)) break;
        if (cp_flags != nullptr) {  // the key block's chunk may still be arriving from its owner
          const int c = (j * BKV) / L;
          const int owner = c < cp_size ? c : 2 * cp_size - 1 - c;
          const long long t0 = clock64();
          bool ok = true;
          while (!cp_flag_ready(cp_flags + owner, cp_epoch)) {
            if (clock64() - t0 > wait_cycles) {
              atomicExch(&g_attn_tc_error, 5);
              *abort_flag = 1;
              ok = false;
              break;
            }
          }
          if (!ok) break;
          asm volatile("fence.proxy.async.global;\n" ::: "memory");
        }
        const int kr = k0 + j * BKV;
        mbar_expect_tx(bar_full + 8 * s, K_BYTES + V_BYTES);
        tma_3d(sK + s * K_BYTES, &tk, bar_full + 8 * s, 0, kvh, kr);
        tma_3d(sK + s * K_BYTES + K_BYTES / 2, &tk, bar_full + 8 * s, 64, kvh, kr);
        tma_3d(sV + s * V_BYTES, &tv, bar_full + 8 * s, 0, kvh, kr);
        tma_3d(sV + s * V_BYTES + V_BYTES / 2, &tv, bar_full + 8 * s, 64, kvh, kr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nblk > 0) {
      bool ok = fwait(bar_q, 0, abort_flag, 2);
      auto issue_s = [&](int j) -> bool {
        const int s = j % STAGES, sb = j & 1;
        if (!fwait(bar_full + 8 * s, (j / STAGES) & 1, abort_flag, 3)) return false;
        if (!fwait(bar_sfree + 8 * sb, ((j >> 1) & 1) ^ 1, abort_flag, 4)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t qa = sQ + (kk >> 2) * (Q_BYTES / 2) + (kk & 3) * 32;
          const uint32_t ka = sK + s * K_BYTES + (kk >> 2) * (K_BYTES / 2) + (kk & 3) * 32;
          umma_bf16(tmem + sb * BKV, desc_kmajor_sw128(qa), desc_kmajor_sw128(ka), IDESC_S, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar_s + 8 * sb);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nblk && ok; ++j) {
        if (j + 1 < nblk && !issue_s(j + 1)) break;
        if (!fwait(bar_p, j & 1, abort_flag, 6)) break;
        tc_fence_after();
        const int s = j % STAGES;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          const uint32_t pa = sK + s * K_BYTES + kk * 32;      // P_j: 128 rows x 64 keys, K-major
          const uint32_t va = sV + s * V_BYTES + kk * 2048;    // V_j: MN-major, 16 keys per step
          umma_bf16(t_o, desc_kmajor_sw128(pa), desc_mn(va), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(bar_o);
        umma_commit(bar_empty + 8 * s);
      }
    }
    __syncwarp();
  } else {
    // softmax warps 2..5: query row = TMEM lane
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qi = m0 + r;  // query index within the segment
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    float m_use = -INFINITY, l = 0.f;
    bool alive = true;
    for (int j = 0; j < nblk && alive; ++j) {
      const int sb = j & 1, s = j % STAGES;
      if (!fwait(bar_s + 8 * sb, (j >> 1) & 1, abort_flag, 7)) {
        alive = false;
        break;
      }
      tc_fence_after();
      float sv[BKV];
      {
        uint32_t u[32];
        tmem_ld32(tmem + lane_off + sb * BKV, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(u[i]);
        tmem_ld32(tmem + lane_off + sb * BKV + 32, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[32 + i] = __uint_as_float(u[i]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree + 8 * sb);
      const int kbase = j * BKV;
      float mb = -INFINITY;
#pragma unroll
      for (int i = 0; i < BKV; ++i) {
        const int key = kbase + i;
        float x = sv[i] * scale_log2;
        if (key >= Lk || (causal && key > qi + off)) x = -INFINITY;
        sv[i] = x;
        mb = fmaxf(mb, x);
      }
      const bool need = mb > m_use + RESCALE_THRESHOLD;
      const float m_new = need ? mb : m_use;
      const float alpha = need ? exp2f(m_use - m_new) : 1.f;  // 0 when m_use was -inf
      const float mref = m_new == -INFINITY ? 0.f : m_new;
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < BKV; ++i) {
        sv[i] = exp2f(sv[i] - mref);
        psum += sv[i];
      }
      // PV_{j-1} must be complete before O is touched (and before it is waited
      // for a second time: every phase of bar_o is observed in order)
      if (j > 0) {
        if (!fwait(bar_o, (j - 1) & 1, abort_flag, 8)) {
          alive = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t u[32];
            tmem_ld32(t_o + lane_off + c * 32, u);
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
            tmem_st32(t_o + lane_off + c * 32, u);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        }
      }
      l = l * alpha + psum;
      m_use = m_new;
      // P_j (bf16) into the K_j slot, K-major 128-byte swizzle: row r, 16-byte chunk c at c ^ (r & 7)
      uint8_t* prow = gbase + Q_BYTES + s * K_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        uint32_t* pv = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 hh = __floats2bfloat162_rn(sv[8 * c + 2 * e], sv[8 * c + 2 * e + 1]);
          pv[e] = *reinterpret_cast<uint32_t*>(&hh);
        }
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p);
    }
    // epilogue: O / l
    if (alive && nblk > 0) {
      if (fwait(bar_o, (nblk - 1) & 1, abort_flag, 9)) {
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const bool store = qi < L;
        __nv_bfloat16* orow = o + ((long long)(s0 + qi) * nq + h) * HD;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t u[32];
          tmem_ld32(t_o + lane_off + c * 32, u);
          if (store) {
            uint4 v[4];
            uint32_t* pv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              __nv_bfloat162 hh =
                  __floats2bfloat162_rn(__uint_as_float(u[2 * e]) * inv, __uint_as_float(u[2 * e + 1]) * inv);
              pv[e] = *reinterpret_cast<uint32_t*>(&hh);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) reinterpret_cast<uint4*>(orow + c * 32)[e] = v[e];
          }
        }
        if (store)
          lse[(long long)h * T_total + s0 + qi] =
              l > 0.f ? m_use * 0.69314718055994531f + logf(l) : -INFINITY;
      }
    } else if (nblk == 0 && qi < L) {
      __nv_bfloat16* orow = o + ((long long)(s0 + qi) * nq + h) * HD;
      for (int d = 0; d < HD; ++d) orow[d] = __float2bfloat16_rn(0.f);
      lse[(long long)h * T_total + s0 + qi] = -INFINITY;
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS));
  }
}


// ============================================================ backward
//
// One CTA per (128-key tile, kv head, sequence): K_t and V_t stay in shared
// memory; the CTA walks every (query head of the group, 64-query block) that
// sees the tile and accumulates dK_t and dV_t in tensor memory, so the group's
// query heads are summed without atomics and dK / dV are written once, as bf16.
// Per step (query block j of head h):
//
//   S^T  = K_t Q_j^T      M=128 keys, N=64 queries, K=128 dims   (A, B K-major)
//   dP^T = V_t dO_j^T     same shape
//   P^T  = exp2(S^T c - lse_j),  dS^T = P^T (dP^T - D_j) * scale  (compute warps,
//          thread = key row; written to shared memory as bf16, K-major)
//   dV  += P^T dO_j       M=128 keys, N=128 dims, K=64 queries    (dO_j read MN-major)
//   dK  += dS^T Q_j       same, Q_j read MN-major
//   dQ_j^T = K_t^T dS^T   M=128 dims, N=64 queries, K=128 keys    (both read MN-major)
//
// The same shared-memory bytes serve both majors: a K-major [rows x 64] tile of
// 128-byte swizzled rows is also the MN-major layout of its transpose (rows = the
// reduction index).  dQ_j^T leaves tensor memory through the compute warps into
// an fp32 [64 x 128] staging tile that one thread adds into the global dQ
// accumulator with a TMA bulk tensor reduce-add (cp.reduce.async.bulk.tensor),
// so partial dQ tiles of different key tiles combine without per-element atomics.
// TMEM: S^T 64 + dP^T 64 + dV 128 + dK 128 + dQ^T 64 columns (512 allocated).
// Shared: K 32 KB + V 32 KB + 2 stages x (Q 16 KB + dO 16 KB) + P^T 16 KB +
// dS^T 16 KB + dQ staging 32 KB + lse/D 512 B.  One CTA per SM.
constexpr int BBQ = 64;                       // queries per step
constexpr int KT_BYTES = 128 * HD * 2;        // 32 KB (K or V tile)
constexpr int QB_BYTES = BBQ * HD * 2;        // 16 KB (Q or dO block)
constexpr int PT_BYTES = 128 * BBQ * 2;       // 16 KB (P^T or dS^T)
constexpr int DQ_BYTES = BBQ * HD * 4;        // 32 KB fp32 staging
constexpr int BWD_SMEM = 2 * KT_BYTES + 2 * 2 * QB_BYTES + 2 * PT_BYTES + DQ_BYTES + 512 + 1024 + 256;
constexpr uint32_t IDESC_ST = idesc_bf16(128, BBQ);                                   // S^T, dP^T
constexpr uint32_t IDESC_DKV = idesc_bf16(128, HD) | (1u << 16);                      // dV, dK: B MN-major
constexpr uint32_t IDESC_DQ = idesc_bf16(128, BBQ) | (1u << 15) | (1u << 16);        // dQ^T: A, B MN-major

__device__ __forceinline__ uint64_t desc_mn_lbo(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }

__global__ void __launch_bounds__(192, 1)
fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                 const __grid_constant__ CUtensorMap tdq, const float* __restrict__ lse, const float* __restrict__ Dv,
                 const int* __restrict__ cu, const int* __restrict__ seg, int nq, int nkv, float scale,
                 float scale_log2, int causal, int T_total, __nv_bfloat16* __restrict__ dk,
                 __nv_bfloat16* __restrict__ dv, float* __restrict__ dk_acc, float* __restrict__ dv_acc) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sK = base;
  const uint32_t sV = sK + KT_BYTES;
  const uint32_t sQ = sV + KT_BYTES;              // stage s: sQ + s * QB_BYTES
  const uint32_t sDO = sQ + 2 * QB_BYTES;         // stage s: sDO + s * QB_BYTES
  const uint32_t sPT = sDO + 2 * QB_BYTES;
  const uint32_t sDS = sPT + PT_BYTES;
  const uint32_t sDQ = sDS + PT_BYTES;
  float* dq_stage = reinterpret_cast<float*>(gbase + (sDQ - base));
  float* lse_s = reinterpret_cast<float*>(gbase + (sDQ - base) + DQ_BYTES);  // [64] (log2 units)
  float* d_s = lse_s + BBQ;                                                  // [64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(gbase + (sDQ - base) + DQ_BYTES + 512);
  const uint32_t bar_kv = smem_u32(bars);
  const uint32_t bar_full = bar_kv + 8;       // [2]
  const uint32_t bar_empty = bar_full + 16;   // [2]
  const uint32_t bar_sdp = bar_empty + 16;    // S^T and dP^T in TMEM
  const uint32_t bar_sfree = bar_sdp + 8;     // compute warps read them (count 4)
  const uint32_t bar_p = bar_sfree + 8;       // P^T and dS^T in shared memory (count 4)
  const uint32_t bar_dq = bar_p + 8;          // dV, dK, dQ^T MMAs of the step complete
  const uint32_t bar_dqfree = bar_dq + 8;     // compute warps read dQ^T (count 4)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x;  // kv head
  const int kt0 = blockIdx.y * 128;
  const int b = blockIdx.z;
  const int s0 = seg ? seg[4 * b] : cu[b];
  const int L = seg ? seg[4 * b + 1] : cu[b + 1] - s0;
  const int k0 = seg ? seg[4 * b + 2] : s0;
  const int Lk = seg ? seg[4 * b + 3] : L;
  const int off = Lk - L;
  if (kt0 >= Lk) return;
  const int G = nq / nkv;
  const int nqb = (L + BBQ - 1) / BBQ;
  // first query block that sees any key of the tile: 64 j + 63 + off >= kt0
  const int jb = causal ? max(0, (kt0 - off - (BBQ - 1) + BBQ - 1) / BBQ) : 0;
  const int per_head = max(0, nqb - jb);
  const int nsteps = G * per_head;

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_sdp, 1);
    mbar_init(bar_sfree, 4);
    mbar_init(bar_p, 4);
    mbar_init(bar_dq, 1);
    mbar_init(bar_dqfree, 4);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(512u));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_dp = tmem + 64, t_dv = tmem + 128, t_dk = tmem + 256, t_dq = tmem + 384;
  auto step_of = [&](int i, int& h, int& j) {
    h = g * G + i / per_head;
    j = jb + i % per_head;
  };

  if (warp == 0) {
    if (lane == 0 && nsteps > 0) {
      mbar_expect_tx(bar_kv, 2 * KT_BYTES);
      tma_3d(sK, &tk, bar_kv, 0, g, k0 + kt0);
      tma_3d(sK + KT_BYTES / 2, &tk, bar_kv, 64, g, k0 + kt0);
      tma_3d(sV, &tv, bar_kv, 0, g, k0 + kt0);
      tma_3d(sV + KT_BYTES / 2, &tv, bar_kv, 64, g, k0 + kt0);
      for (int i = 0; i < nsteps && !*abort_flag; ++i) {
        const int s = i & 1;
        if (!fwait(bar_empty + 8 * s, ((i >> 1) & 1) ^ 1, abort_flag, 11)) break;
        int h, j;
        step_of(i, h, j);
        const int qr = s0 + j * BBQ;
        mbar_expect_tx(bar_full + 8 * s, 2 * QB_BYTES);
        tma_3d(sQ + s * QB_BYTES, &tq, bar_full + 8 * s, 0, h, qr);
        tma_3d(sQ + s * QB_BYTES + QB_BYTES / 2, &tq, bar_full + 8 * s, 64, h, qr);
        tma_3d(sDO + s * QB_BYTES, &tdo, bar_full + 8 * s, 0, h, qr);
        tma_3d(sDO + s * QB_BYTES + QB_BYTES / 2, &tdo, bar_full + 8 * s, 64, h, qr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nsteps > 0) {
      bool ok = fwait(bar_kv, 0, abort_flag, 12);
      // S^T / dP^T of step i+1 are issued as soon as the compute warps have read
      // step i's (single TMEM buffer), ahead of step i's dV / dK / dQ MMAs: the
      // tensor core computes them while the compute warps form P^T and dS^T.
      auto issue_sdp = [&](int i) -> bool {
        const int s = i & 1;
        if (!fwait(bar_full + 8 * s, (i >> 1) & 1, abort_flag, 13)) return false;
        tc_fence_after();
        const uint32_t q0 = sQ + s * QB_BYTES, o0 = sDO + s * QB_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * (KT_BYTES / 2) + (kk & 3) * 32;
          const uint32_t qo = (kk >> 2) * (QB_BYTES / 2) + (kk & 3) * 32;
          umma_bf16(t_s, desc_kmajor_sw128(sK + ko), desc_kmajor_sw128(q0 + qo), IDESC_ST, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t ko = (kk >> 2) * (KT_BYTES / 2) + (kk & 3) * 32;
          const uint32_t qo = (kk >> 2) * (QB_BYTES / 2) + (kk & 3) * 32;
          umma_bf16(t_dp, desc_kmajor_sw128(sV + ko), desc_kmajor_sw128(o0 + qo), IDESC_ST, kk > 0 ? 1u : 0u);
        }
        umma_commit(bar_sdp);
        return true;
      };
      if (ok) ok = issue_sdp(0);
      for (int i = 0; i < nsteps && ok; ++i) {
        const int s = i & 1;
        if (i + 1 < nsteps) {
          if (!fwait(bar_sfree, i & 1, abort_flag, 14)) break;
          if (!issue_sdp(i + 1)) break;
        }
        if (!fwait(bar_p, i & 1, abort_flag, 15)) break;
        if (!fwait(bar_dqfree, (i & 1) ^ 1, abort_flag, 16)) break;
        tc_fence_after();
        const uint32_t q0 = sQ + s * QB_BYTES, o0 = sDO + s * QB_BYTES;
#pragma unroll
        for (int kk = 0; kk < BBQ / 16; ++kk) {  // reduce over the 64 queries
          umma_bf16(t_dv, desc_kmajor_sw128(sPT + kk * 32), desc_mn_lbo(o0 + kk * 2048, QB_BYTES / 2), IDESC_DKV,
                    (i > 0 || kk > 0) ? 1u : 0u);
          umma_bf16(t_dk, desc_kmajor_sw128(sDS + kk * 32), desc_mn_lbo(q0 + kk * 2048, QB_BYTES / 2), IDESC_DKV,
                    (i > 0 || kk > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk)  // reduce over the 128 keys
          umma_bf16(t_dq, desc_mn_lbo(sK + kk * 2048, KT_BYTES / 2), desc_mn_lbo(sDS + kk * 2048, 8192u), IDESC_DQ,
                    kk > 0 ? 1u : 0u);
        umma_commit(bar_dq);
        umma_commit(bar_empty + 8 * s);
      }
    }
    __syncwarp();
  } else {
    // compute warps: TMEM lane = key row of the tile (S^T, dP^T, dV, dK) or dim (dQ^T)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int ct = threadIdx.x - 64;  // 0..127
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    const int kg = kt0 + r;  // key index within the sequence's keys
    bool alive = nsteps > 0;
    bool issued = false;  // a TMA reduce of the staging tile may be in flight (thread ct == 0)
    // Every compute warp executes the same sequence of named barriers (bar 1) whatever
    // happens to its waits: after a failed wait a warp skips the work but keeps
    // stepping, so no warp is left at a named barrier (which cannot time out).
    auto drain_dq = [&](int i, bool live) -> bool {  // dQ^T of step i: TMEM -> staging -> reduce-add
      const bool ok = live && fwait(bar_dq, i & 1, abort_flag, 17);
      if (ok) tc_fence_after();
      int h, j;
      step_of(i, h, j);
      if (ct == 0 && issued) asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
      bar_compute();
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < BBQ / 32; ++c) {
          uint32_t u[32];
          tmem_ld32(t_dq + lo + c * 32, u);
#pragma unroll
          for (int e = 0; e < 32; ++e) dq_stage[(c * 32 + e) * HD + r] = __uint_as_float(u[e]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_dqfree);
      }
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      bar_compute();
      if (ct == 0 && ok && !*abort_flag) {
        asm volatile(
            "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];\n" ::"l"(
                &tdq),
            "r"(sDQ), "r"(0), "r"(h), "r"(s0 + j * BBQ)
            : "memory");
        asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
        issued = true;
      }
      return ok;
    };
    for (int i = 0; i < nsteps; ++i) {
      int h, j;
      step_of(i, h, j);
      // this step's lse (log2 units) and D rows
      bar_compute();
      if (ct < BBQ) {
        const int q = j * BBQ + ct;
        lse_s[ct] = q < L ? lse[(long long)h * T_total + s0 + q] * 1.4426950408889634f : 0.f;
      } else {
        const int q = j * BBQ + ct - BBQ;
        d_s[ct - BBQ] = q < L ? Dv[(long long)h * T_total + s0 + q] : 0.f;
      }
      bar_compute();
      float sv[BBQ], pv[BBQ];
      const bool ok = alive && fwait(bar_sdp, i & 1, abort_flag, 18);
      if (ok) {
        tc_fence_after();
        uint32_t u[32];
        tmem_ld32(t_s + lo, u);
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[e] = __uint_as_float(u[e]);
        tmem_ld32(t_s + lo + 32, u);
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[32 + e] = __uint_as_float(u[e]);
        tmem_ld32(t_dp + lo, u);
#pragma unroll
        for (int e = 0; e < 32; ++e) pv[e] = __uint_as_float(u[e]);
        tmem_ld32(t_dp + lo + 32, u);
#pragma unroll
        for (int e = 0; e < 32; ++e) pv[32 + e] = __uint_as_float(u[e]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_sfree);
#pragma unroll
        for (int c = 0; c < BBQ; ++c) {
          const int q = j * BBQ + c;
          const bool valid = kg < Lk && q < L && (!causal || kg <= q + off);
          const float p = valid ? exp2f(sv[c] * scale_log2 - lse_s[c]) : 0.f;
          sv[c] = p;
          pv[c] = p * (pv[c] - d_s[c]) * scale;
        }
      }
      alive = ok;
      // the previous step's MMAs read P^T / dS^T: drain its dQ (and so wait for them) first
      if (i > 0) alive = drain_dq(i - 1, alive) && alive;
      if (alive) {
        uint8_t* prow = gbase + (sPT - base) + r * 128;
        uint8_t* drow = gbase + (sDS - base) + r * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 a, d;
          uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
          uint32_t* pd = reinterpret_cast<uint32_t*>(&d);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 x = __floats2bfloat162_rn(sv[8 * c + 2 * e], sv[8 * c + 2 * e + 1]);
            __nv_bfloat162 y = __floats2bfloat162_rn(pv[8 * c + 2 * e], pv[8 * c + 2 * e + 1]);
            pa[e] = *reinterpret_cast<uint32_t*>(&x);
            pd[e] = *reinterpret_cast<uint32_t*>(&y);
          }
          const int pos = (c ^ (r & 7)) << 4;
          *reinterpret_cast<uint4*>(prow + pos) = a;
          *reinterpret_cast<uint4*>(drow + pos) = d;
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_p);
      }
    }
    if (nsteps > 0) alive = drain_dq(nsteps - 1, alive);
    // dK, dV rows of the tile (complete with the last step's commit)
    const bool store = kg < Lk;
    __nv_bfloat16* dkr = dk + ((long long)(k0 + kg) * nkv + g) * HD;
    __nv_bfloat16* dvr = dv + ((long long)(k0 + kg) * nkv + g) * HD;
    if (alive && nsteps > 0) {
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const uint32_t src = half == 0 ? t_dv : t_dk;
        __nv_bfloat16* dst = half == 0 ? dvr : dkr;
        float* acc = half == 0 ? dv_acc : dk_acc;
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t u[32];
          tmem_ld32(src + lo + c * 32, u);
          if (store && acc != nullptr) {
            // segments that share keys (context parallelism) add into fp32 rows
            float4* ar = reinterpret_cast<float4*>(acc + ((long long)(k0 + kg) * nkv + g) * HD + c * 32);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              atomicAdd(ar + e, make_float4(__uint_as_float(u[4 * e]), __uint_as_float(u[4 * e + 1]),
                                            __uint_as_float(u[4 * e + 2]), __uint_as_float(u[4 * e + 3])));
          } else if (store) {
            uint4 v[4];
            uint32_t* pvv = reinterpret_cast<uint32_t*>(v);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              __nv_bfloat162 x = __floats2bfloat162_rn(__uint_as_float(u[2 * e]), __uint_as_float(u[2 * e + 1]));
              pvv[e] = *reinterpret_cast<uint32_t*>(&x);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) reinterpret_cast<uint4*>(dst + c * 32)[e] = v[e];
          }
        }
      }
    } else if (store && nsteps == 0 && dk_acc == nullptr) {
      for (int d = 0; d < HD; ++d) {
        dkr[d] = __float2bfloat16_rn(0.f);
        dvr[d] = __float2bfloat16_rn(0.f);
      }
    }
    if (ct == 0 && issued) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512u));
  }
}

// D[h][t] = sum_d dO[t][h][d] * O[t][h][d] (fp32), one warp per (t, h)
__global__ void fa_bwd_rowdot_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                     long long rows, int nq, int T, float* __restrict__ D) {
  const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const uint2 a = reinterpret_cast<const uint2*>(dout + w * HD)[lane];
  const uint2 c = reinterpret_cast<const uint2*>(out + w * HD)[lane];
  const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
  const __nv_bfloat162* pc = reinterpret_cast<const __nv_bfloat162*>(&c);
  float acc = 0.f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float2 x = __bfloat1622float2(pa[e]), y = __bfloat1622float2(pc[e]);
    acc += x.x * y.x + x.y * y.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const long long t = w / nq;
    const int h = (int)(w % nq);
    D[(long long)h * T + t] = acc;
  }
}

}  // namespace fa
}  // namespace rlb

using namespace rlb;

namespace {

// [T, heads, 128] bf16 view (token stride `ts` elements) as a 3-D tensor map
// {dim, head, token} with a 64 x 1 x `rows` box, 128-byte swizzle.
CUtensorMap head_tmap(const at::Tensor& x, int rows) {
  CUtensorMap m;
  const int T = x.size(0), H = x.size(1);
  cuuint64_t dims[3] = {(cuuint64_t)fa::HD, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)x.stride(1) * 2, (cuuint64_t)x.stride(0) * 2};
  cuuint32_t box[3] = {64u, 1u, (cuuint32_t)rows};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x.data_ptr(), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "rl_b200 attention (tcgen05): cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

void check_view(const at::Tensor& x, const char* name) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3 && x.scalar_type() == at::kBFloat16 && x.size(2) == fa::HD,
              "rl_b200 attention (tcgen05): ", name, " must be a bf16 CUDA [T, heads, 128] tensor");
  TORCH_CHECK(x.stride(2) == 1 && x.stride(1) == fa::HD && x.stride(0) % 8 == 0 &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "rl_b200 attention (tcgen05): ", name, " needs contiguous heads and 16-byte aligned rows");
}

void launch_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const int* cu, const int* seg, int nseg,
               int max_q, float scale_log2, bool causal, at::Tensor& o, at::Tensor& lse, const uint32_t* cp_flags,
               uint32_t cp_epoch, int cp_size) {
  const int nq = q.size(1), nkv = k.size(1), T_ = q.size(0);
  const CUtensorMap tq = head_tmap(q, fa::BQ);
  const CUtensorMap tk = head_tmap(k, fa::BKV);
  const CUtensorMap tv = head_tmap(v, fa::BKV);
  auto kern = fa::fa_fwd_tc_kernel;
  RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::SMEM));
  dim3 grid(nq, (max_q + fa::BQ - 1) / fa::BQ, nseg);
  kern<<<grid, 192, fa::SMEM, stream()>>>(tq, tk, tv, cu, nq, nkv, scale_log2, causal ? 1 : 0,
                                          (__nv_bfloat16*)o.data_ptr(), lse.data_ptr<float>(), T_, seg, cp_flags,
                                          cp_epoch, cp_size, (long long)peer_wait_cycles());
  RLB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

// Same contract as flash_attn_fwd (head dim 128): o [T, nq, 128] bf16, lse [nq, T]
// fp32 (natural log of the softmax denominator of the scaled scores).
std::vector<at::Tensor> flash_attn_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                          int64_t max_seqlen, double scale, bool causal) {
  check_view(q, "q");
  check_view(k, "k");
  check_view(v, "v");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T_ = q.size(0), nq = q.size(1), nkv = k.size(1);
  TORCH_CHECK(nq % nkv == 0, "rl_b200 attention: nq must be a multiple of nkv");
  auto cu = cu_seqlens.to(at::kInt).contiguous();
  const int B = cu.size(0) - 1;
  auto o = at::empty({T_, nq, fa::HD}, q.options());
  auto lse = at::empty({nq, T_}, q.options().dtype(at::kFloat));
  if (T_ == 0 || B == 0 || max_seqlen == 0) return {o, lse};
  launch_tc(q, k, v, cu.data_ptr<int>(), nullptr, B, (int)max_seqlen, (float)(scale * 1.4426950408889634), causal, o,
            lse, nullptr, 0u, 0);
  return {o, lse};
}

// Segment form (context parallelism), same contract as flash_attn_seg_fwd.
std::vector<at::Tensor> flash_attn_seg_fwd_tc(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor seg, int64_t max_q,
                                              double scale, c10::optional<at::Tensor> cp_flags, int64_t cp_epoch,
                                              int64_t cp_size) {
  check_view(q, "q");
  check_view(k, "k");
  check_view(v, "v");
  TORCH_CHECK(seg.is_cuda() && seg.scalar_type() == at::kInt && seg.dim() == 2 && seg.size(1) == 4 &&
                  seg.is_contiguous(),
              "rl_b200 segment attention: seg int32 [S, 4]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T_ = q.size(0), nq = q.size(1);
  const int S = seg.size(0);
  auto o = at::zeros({T_, nq, fa::HD}, q.options());
  auto lse = at::zeros({nq, T_}, q.options().dtype(at::kFloat));
  if (T_ == 0 || S == 0 || max_q == 0) return {o, lse};
  launch_tc(q, k, v, nullptr, seg.data_ptr<int>(), S, (int)max_q, (float)(scale * 1.4426950408889634), true, o, lse,
            cp_flags ? reinterpret_cast<const uint32_t*>(cp_flags->data_ptr<int>()) : nullptr, (uint32_t)cp_epoch,
            (int)cp_size);
  return {o, lse};
}


namespace {

// fp32 [T, heads, 128] accumulator as a 3-D tensor map with a 128 x 1 x 64 box
// (no swizzle; the staging tile is [64 rows][128 floats]) for the bulk reduce-add.
CUtensorMap dq_tmap(const at::Tensor& x) {
  CUtensorMap m;
  const int T = x.size(0), H = x.size(1);
  cuuint64_t dims[3] = {(cuuint64_t)fa::HD, (cuuint64_t)H, (cuuint64_t)T};
  cuuint64_t strides[2] = {(cuuint64_t)x.stride(1) * 4, (cuuint64_t)x.stride(0) * 4};
  cuuint32_t box[3] = {(cuuint32_t)fa::HD, 1u, (cuuint32_t)fa::BBQ};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, x.data_ptr(), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "rl_b200 attention bwd (tcgen05): cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

std::vector<at::Tensor> bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                               at::Tensor lse, const int* cu, const int* seg, int nseg, int max_k, double scale,
                               bool causal, bool accumulate_kv) {
  check_view(q, "q");
  check_view(k, "k");
  check_view(v, "v");
  check_view(dout, "dout");
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous(), "rl_b200 attention bwd: dout / out must be contiguous");
  const int T_ = q.size(0), nq = q.size(1), nkv = k.size(1), Tk = k.size(0);
  TORCH_CHECK(nq % nkv == 0, "rl_b200 attention: nq must be a multiple of nkv");
  auto dq_acc = at::zeros({T_, nq, fa::HD}, q.options().dtype(at::kFloat));
  auto dk = at::zeros({Tk, nkv, fa::HD}, q.options());
  auto dv = at::zeros({Tk, nkv, fa::HD}, q.options());
  at::Tensor dk_acc, dv_acc;
  if (accumulate_kv) {
    dk_acc = at::zeros({Tk, nkv, fa::HD}, q.options().dtype(at::kFloat));
    dv_acc = at::zeros({Tk, nkv, fa::HD}, q.options().dtype(at::kFloat));
  }
  if (T_ == 0 || nseg == 0 || max_k == 0) return {dq_acc.to(q.scalar_type()), dk, dv};
  auto D = at::empty({nq, T_}, q.options().dtype(at::kFloat));
  const long long rows = (long long)T_ * nq;
  fa::fa_bwd_rowdot_kernel<<<(int)((rows * 32 + 255) / 256), 256, 0, stream()>>>(
      (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)out.data_ptr(), rows, nq, T_, D.data_ptr<float>());
  const CUtensorMap tq = head_tmap(q, fa::BBQ);
  const CUtensorMap tk = head_tmap(k, 128);
  const CUtensorMap tv = head_tmap(v, 128);
  const CUtensorMap tdo = head_tmap(dout, fa::BBQ);
  const CUtensorMap tdq = dq_tmap(dq_acc);
  auto kern = fa::fa_bwd_tc_kernel;
  RLB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, fa::BWD_SMEM));
  dim3 grid(nkv, (max_k + 127) / 128, nseg);
  kern<<<grid, 192, fa::BWD_SMEM, stream()>>>(tq, tk, tv, tdo, tdq, lse.data_ptr<float>(), D.data_ptr<float>(), cu,
                                             seg, nq, nkv, (float)scale, (float)(scale * 1.4426950408889634),
                                             causal ? 1 : 0, T_, (__nv_bfloat16*)dk.data_ptr(),
                                             (__nv_bfloat16*)dv.data_ptr(),
                                             accumulate_kv ? dk_acc.data_ptr<float>() : nullptr,
                                             accumulate_kv ? dv_acc.data_ptr<float>() : nullptr);
  RLB_CUDA_CHECK(cudaGetLastError());
  if (accumulate_kv) return {dq_acc.to(q.scalar_type()), dk_acc.to(q.scalar_type()), dv_acc.to(q.scalar_type())};
  return {dq_acc.to(q.scalar_type()), dk, dv};
}

}  // namespace

// Same contract as flash_attn_bwd (head dim 128): {dq, dk, dv}, bf16.
std::vector<at::Tensor> flash_attn_bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                                          at::Tensor lse, at::Tensor cu_seqlens, int64_t max_seqlen, double scale,
                                          bool causal) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto cu = cu_seqlens.to(at::kInt).contiguous();
  return bwd_tc(dout, q, k, v, out, lse, cu.data_ptr<int>(), nullptr, cu.size(0) - 1, (int)max_seqlen, scale, causal,
                false);
}

// Segment form (context parallelism), same contract as flash_attn_seg_bwd.
std::vector<at::Tensor> flash_attn_seg_bwd_tc(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v,
                                              at::Tensor out, at::Tensor lse, at::Tensor seg, int64_t max_k,
                                              double scale) {
  TORCH_CHECK(seg.is_cuda() && seg.scalar_type() == at::kInt && seg.dim() == 2 && seg.size(1) == 4 &&
                  seg.is_contiguous(),
              "rl_b200 segment attention: seg int32 [S, 4]");
  const c10::cuda::CUDAGuard guard(q.device());
  return bwd_tc(dout, q, k, v, out, lse, nullptr, seg.data_ptr<int>(), seg.size(0), (int)max_k, scale, true, true);
}

int64_t attn_tc_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, fa::g_attn_tc_error, sizeof(int)));
  if (reset) {
    int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(fa::g_attn_tc_error, &z, sizeof(int)));
  }
  return v;
}
