// Attention kernels.
//
// 1. paged_decode_attn: one query token per sequence against its paged KV
//    history (rollout decode).  Grid (B, nkv, splits); a CTA serves all G query
//    heads of one KV head, so every K/V byte is read once per group.  Lanes own
//    tokens for the Q.K dot products and own head dims for the P.V update; the
//    split-K partials (o, m, l) are merged by a second kernel.
// 2. flash_attn_fwd: packed variable-length causal GQA attention (training
//    forward and prompt prefill).  64-query x 64-key tiles, 4 warps, double-
//    buffered cp.async K/V tiles in XOR-swizzled shared memory, ldmatrix
//    fragments, bf16 mma.sync with fp32 accumulators, online softmax in base 2.
// 3. flash_attn_bwd: per CTA one KV head and 64 keys; loops over the group's
//    query heads and 32-query blocks, accumulating dK/dV in registers; dQ is
//    accumulated with vector fp32 atomics into a scratch buffer and converted
//    (scaled, cast) by a final kernel.
#include "common.cuh"

namespace rlb {

typedef __nv_bfloat16 bf16;

// ----------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

__device__ __forceinline__ void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Tile of R rows x (CH * 8) bf16 in shared memory, 16-byte chunks XOR-swizzled so
// that 8 consecutive rows at one logical chunk hit 8 distinct bank groups.
template <int CH>
__device__ __forceinline__ int swz(int row, int ch) {
  if constexpr (CH >= 8) return row * CH + (ch ^ (row & 7));
  else if constexpr (CH == 4) return row * CH + (ch ^ ((row >> 1) & 3));
  else if constexpr (CH == 2) return row * CH + (ch ^ ((row >> 2) & 1));
  else return row * CH + ch;
}

template <int CH>
__device__ __forceinline__ void load_tile(bf16* s, const bf16* g, long long row_stride, int rows, int rows_valid,
                                          int tid, int nthr) {
  for (int c = tid; c < rows * CH; c += nthr) {
    const int r = c / CH, ch = c % CH;
    const bool ok = r < rows_valid;
    const bf16* src = g + (long long)(ok ? r : 0) * row_stride + ch * 8;
    cp_async16(smem_u32(s + swz<CH>(r, ch) * 8), src, ok ? 16 : 0);
  }
}

__device__ int g_attn_error = 0;

// Bounded wait (at most `limit` cycles) until *p >= v; false on expiry.
__device__ __forceinline__ bool cp_wait_flag(const uint32_t* p, uint32_t v, long long limit) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t x;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(x) : "l"(p) : "memory");
    if ((int)(x - v) >= 0) return true;
    if (clock64() - t0 > limit) return false;
  }
}

// ============================================================ decode attention
template <typename C, int HD, int G>
__global__ void __launch_bounds__(128)
paged_decode_kernel(const bf16* __restrict__ q, long long q_stride, const C* __restrict__ kc,
                    const C* __restrict__ vc, const int* __restrict__ block_tables, int max_blocks,
                    const int* __restrict__ seq_lens, int block_size, int nkv, float scale_log2, float k_scale,
                    float v_scale, int tokens_per_split, float* __restrict__ part_o, float* __restrict__ part_ml,
                    bf16* __restrict__ out) {
  constexpr int DPL = HD / 32;  // dims per lane in the P.V phase
  pdl_launch_dependents();
  __shared__ float qs[G][HD];
  __shared__ float red_m[4][G], red_l[4][G];
  __shared__ float red_o[4][G][HD];
  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int L = seq_lens[b];
  const int t_begin = split * tokens_per_split;
  const int t_end = min(L, t_begin + tokens_per_split);
  const int nq = nkv * G;
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int g = e / HD, d = e % HD;
    qs[g][d] = __bfloat162float(q[(long long)b * q_stride + (kvh * G + g) * HD + d]) * scale_log2;
  }
  __syncthreads();
  float m[G], l[G], o[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) o[g][i] = 0.f;
  }
  const int* bt = block_tables + (long long)b * max_blocks;
  for (int base = t_begin + w * 32; base < t_end; base += 128) {
    const int t = base + lane;
    float s[G];
    const bool live = t < t_end;
    long long row = 0;
    if (live) {
      const int blk = bt[t / block_size];
      row = ((long long)blk * block_size + (t % block_size)) * nkv + kvh;
      const C* kr = kc + row * HD;
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll 4
      for (int d0 = 0; d0 < HD; d0 += 8) {
        float kf[8];
        if constexpr (std::is_same<C, bf16>::value) {
          unpack8(*reinterpret_cast<const bf16x8*>(kr + d0), kf);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) kf[i] = float(kr[d0 + i]) * k_scale;
        }
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int i = 0; i < 8; ++i) s[g] += qs[g][d0 + i] * kf[i];
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = -INFINITY;
    }
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mx = warp_max(s[g]);
      const float mn = fmaxf(m[g], mx);
      const float alpha = exp2f(m[g] - mn);
      p[g] = live ? exp2f(s[g] - mn) : 0.f;
      l[g] = l[g] * alpha + warp_sum(p[g]);
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[g][i] *= alpha;
      m[g] = mn;
    }
    const int ntok = min(32, t_end - base);
    for (int j = 0; j < ntok; ++j) {
      const long long rj = __shfl_sync(0xffffffffu, row, j);
      const C* vr = vc + rj * HD + lane * DPL;
      float vf[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        if constexpr (std::is_same<C, bf16>::value) vf[i] = __bfloat162float(vr[i]);
        else vf[i] = float(vr[i]) * v_scale;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pj = __shfl_sync(0xffffffffu, p[g], j);
#pragma unroll
        for (int i = 0; i < DPL; ++i) o[g][i] += pj * vf[i];
      }
    }
  }
  // merge the 4 warps
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      red_m[w][g] = m[g];
      red_l[w][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int i = 0; i < DPL; ++i) red_o[w][g][lane * DPL + i] = o[g][i];
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int g = e / HD, d = e % HD;
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < 4; ++k) M = fmaxf(M, red_m[k][g]);
    float Lsum = 0.f, O = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float f = red_m[k][g] == -INFINITY ? 0.f : exp2f(red_m[k][g] - M);
      Lsum += red_l[k][g] * f;
      O += red_o[k][g][d] * f;
    }
    const int h = kvh * G + g;
    if (part_o == nullptr) {
      out[(long long)b * nq * HD + h * HD + d] = __float2bfloat16_rn(Lsum > 0.f ? O / Lsum : 0.f);
    } else {
      const long long pi = ((long long)(b * nq + h) * gridDim.z + split);
      part_o[pi * HD + d] = O;
      if (d == 0) {
        part_ml[pi * 2] = M;
        part_ml[pi * 2 + 1] = Lsum;
      }
    }
  }
}

// Tensor-core decode: each warp owns 32-token K/V tiles of one (sequence, KV
// head), loaded with cp.async as whole 256-byte rows (coalesced) into swizzled
// shared memory; S = Q K^T and O += P V run as m16n8k16 MMAs with the G query
// heads of the group in rows 0..G-1 of the A operand (rows G..15 are zero).
// The 4 warps of a CTA take tiles round-robin and merge their online-softmax
// states at the end; split-K partials go to the combine kernel.
template <int HD, int G>
__global__ void __launch_bounds__(128)
paged_decode_tc_kernel(const bf16* __restrict__ q, long long q_stride, const bf16* __restrict__ kc,
                       const bf16* __restrict__ vc, const int* __restrict__ block_tables, int max_blocks,
                       const int* __restrict__ seq_lens, int block_size, int nkv, float scale_log2,
                       int tokens_per_split, float* __restrict__ part_o, float* __restrict__ part_ml,
                       bf16* __restrict__ out) {
  constexpr int BT = 32, CH = HD / 8, KS = HD / 16, NT = HD / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  bf16* Ks = reinterpret_cast<bf16*>(smem_raw) + w * 2 * BT * HD;
  bf16* Vs = Ks + BT * HD;
  float* red = reinterpret_cast<float*>(reinterpret_cast<bf16*>(smem_raw) + 4 * 2 * BT * HD);  // [4][G][HD+2]
  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int g = lane >> 2, t = lane & 3;
  const int L = seq_lens[b];
  const int t_begin = split * tokens_per_split;
  const int t_end = min(L, t_begin + tokens_per_split);
  const int nq = nkv * G;
  const int* bt = block_tables + (long long)b * max_blocks;
  // Q fragments (rows >= G are zero)
  uint32_t qf[KS][4];
  {
    const bf16* qb = q + (long long)b * q_stride + (long long)kvh * G * HD;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int c0 = kk * 16 + 2 * t;
      const bool ok = g < G;
      const uint32_t lo0 = ok ? *reinterpret_cast<const uint32_t*>(qb + g * HD + c0) : 0u;
      const uint32_t lo1 = ok ? *reinterpret_cast<const uint32_t*>(qb + g * HD + c0 + 8) : 0u;
      qf[kk][0] = lo0;
      qf[kk][1] = 0u;  // row g + 8 >= 8 > G - 1 for G <= 8
      qf[kk][2] = lo1;
      qf[kk][3] = 0u;
    }
  }
  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  float mrow = -INFINITY, lrow = 0.f;
  for (int t0 = t_begin + w * BT; t0 < t_end; t0 += 4 * BT) {
    const int nvalid = min(BT, t_end - t0);
    // cp.async K/V rows of this tile (per-row block-table lookup)
    for (int c = lane; c < BT * CH; c += 32) {
      const int r = c / CH, ch = c % CH;
      const bool ok = r < nvalid;
      long long row = 0;
      if (ok) {
        const int tok = t0 + r;
        row = ((long long)bt[tok / block_size] * block_size + (tok % block_size)) * nkv + kvh;
      }
      cp_async16(smem_u32(Ks + swz<CH>(r, ch) * 8), kc + row * HD + ch * 8, ok ? 16 : 0);
      cp_async16(smem_u32(Vs + swz<CH>(r, ch) * 8), vc + row * HD + ch * 8, ok ? 16 : 0);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncwarp();
    float s[BT / 8][4];
#pragma unroll
    for (int j = 0; j < BT / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int np = 0; np < BT / 16; ++np) {
        uint32_t bfr[4];
        ldsm_x4(bfr, smem_u32(Ks + swz<CH>(np * 16 + ((lane >> 4) << 3) + (lane & 7), 2 * kk + ((lane >> 3) & 1)) * 8));
        mma16816(s[2 * np], qf[kk], bfr[0], bfr[1]);
        mma16816(s[2 * np + 1], qf[kk], bfr[2], bfr[3]);
      }
    }
    // online softmax over row g (rows g+8 are padding)
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < BT / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = 8 * j + 2 * t + e;
        const float v = key < nvalid ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = v;
        mx = fmaxf(mx, v);
      }
      s[j][2] = s[j][3] = 0.f;
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(mrow, mx);
    const float muse = mnew == -INFINITY ? 0.f : mnew;
    const float alpha = exp2f(mrow - muse);
    mrow = mnew;
    lrow *= alpha;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      oacc[j][0] *= alpha;
      oacc[j][1] *= alpha;
    }
#pragma unroll
    for (int j = 0; j < BT / 8; ++j) {
      s[j][0] = exp2f(s[j][0] - muse);
      s[j][1] = exp2f(s[j][1] - muse);
      lrow += s[j][0] + s[j][1];
    }
#pragma unroll
    for (int kk = 0; kk < BT / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = 0u;
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = 0u;
#pragma unroll
      for (int dp = 0; dp < NT / 2; ++dp) {
        uint32_t bfr[4];
        ldsm_x4_t(bfr, smem_u32(Vs + swz<CH>(kk * 16 + (lane & 15), 2 * dp + (lane >> 4)) * 8));
        mma16816(oacc[2 * dp], a, bfr[0], bfr[1]);
        mma16816(oacc[2 * dp + 1], a, bfr[2], bfr[3]);
      }
    }
    __syncwarp();
  }
  lrow += __shfl_xor_sync(0xffffffffu, lrow, 1);
  lrow += __shfl_xor_sync(0xffffffffu, lrow, 2);
  // per-warp state -> shared memory: red[w][g][0..HD) = o, [HD] = m, [HD+1] = l
  constexpr int RS = HD + 2;
  if (g < G) {
    float* rw = red + ((size_t)w * G + g) * RS;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      rw[8 * j + 2 * t] = oacc[j][0];
      rw[8 * j + 2 * t + 1] = oacc[j][1];
    }
    if (t == 0) {
      rw[HD] = mrow;
      rw[HD + 1] = lrow;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += blockDim.x) {
    const int gg = e / HD, d = e % HD;
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < 4; ++k) M = fmaxf(M, red[((size_t)k * G + gg) * RS + HD]);
    float Lsum = 0.f, O = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float* rk = red + ((size_t)k * G + gg) * RS;
      const float f = rk[HD] == -INFINITY ? 0.f : exp2f(rk[HD] - M);
      Lsum += rk[HD + 1] * f;
      O += rk[d] * f;
    }
    const int h = kvh * G + gg;
    if (part_o == nullptr) {
      out[(long long)b * nq * HD + h * HD + d] = __float2bfloat16_rn(Lsum > 0.f ? O / Lsum : 0.f);
    } else {
      const long long pi = ((long long)(b * nq + h) * gridDim.z + split);
      part_o[pi * HD + d] = O;
      if (d == 0) {
        part_ml[pi * 2] = M;
        part_ml[pi * 2 + 1] = Lsum;
      }
    }
  }
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Pipelined tensor-core decode.  Each of the W warps of a CTA streams its own
// sequence of 16-token K/V tiles (tiles w, w+W, w+2W, ... of the CTA's token
// range) through a private ST-stage cp.async ring, so ST-1 tiles per warp are
// always in flight while the warp runs the MMAs of the current one; the
// CTA's block-table entries are staged in shared memory once, so no load on
// the critical path waits for a block-table read.  S = Q K^T and O += P V run
// as m16n8k16 MMAs with the G query heads of the group in rows 0..G-1.  After
// the loop the ring is reused to merge the warps' online-softmax states.
// Requires block_size % 16 == 0 and tokens_per_split % 16 == 0.
template <int HD, int G, int W, int ST>
__global__ void __launch_bounds__(W * 32)
paged_decode_pipe_kernel(const bf16* __restrict__ q, long long q_stride, const bf16* __restrict__ kc,
                         const bf16* __restrict__ vc, const int* __restrict__ block_tables, int max_blocks,
                         const int* __restrict__ seq_lens, int block_size, int nkv, float scale_log2,
                         int tokens_per_split, float* __restrict__ part_o, float* __restrict__ part_ml,
                         bf16* __restrict__ out, int n_blocks) {
  constexpr int BT = 16, CH = HD / 8, KS = HD / 16, NT = HD / 8, TILE = BT * HD;
  pdl_launch_dependents();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  bf16* ring = reinterpret_cast<bf16*>(smem_raw) + (size_t)w * ST * 2 * TILE;
  int* sbt = reinterpret_cast<int*>(smem_raw + (size_t)W * ST * 2 * TILE * sizeof(bf16));
  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int g = lane >> 2, t = lane & 3;
  const int L = seq_lens[b];
  const int t_begin = split * tokens_per_split;
  const int t_end = min(L, t_begin + tokens_per_split);
  const int nq = nkv * G;
  const int* bt = block_tables + (long long)b * max_blocks;
  const int blk0 = t_begin / block_size;
  if (t_end > t_begin) {
    const int nblk = (t_end - 1) / block_size - blk0 + 1;
    for (int i = threadIdx.x; i < nblk; i += W * 32) {
      const int blk = bt[blk0 + i];
      sbt[i] = RLB_IN_BOUNDS(blk, n_blocks, kBoundsBlockTable) ? blk : 0;
    }
  }
  uint32_t qf[KS][4];
  {
    const bf16* qb = q + (long long)b * q_stride + (long long)kvh * G * HD;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int c0 = kk * 16 + 2 * t;
      const bool ok = g < G;
      qf[kk][0] = ok ? *reinterpret_cast<const uint32_t*>(qb + g * HD + c0) : 0u;
      qf[kk][1] = 0u;
      qf[kk][2] = ok ? *reinterpret_cast<const uint32_t*>(qb + g * HD + c0 + 8) : 0u;
      qf[kk][3] = 0u;
    }
  }
  __syncthreads();
  const int ntiles = t_end > t_begin ? (t_end - t_begin + BT - 1) / BT : 0;
  const int n_my = ntiles > w ? (ntiles - w + W - 1) / W : 0;
  auto issue = [&](int k) {
    if (k < n_my) {
      const int t0 = t_begin + (w + k * W) * BT;
      const int nvalid = min(BT, t_end - t0);
      const long long base = (long long)sbt[t0 / block_size - blk0] * block_size + (t0 % block_size);
      bf16* Ks = ring + (k % ST) * 2 * TILE;
      bf16* Vs = Ks + TILE;
#pragma unroll
      for (int c = lane; c < BT * CH; c += 32) {
        const int r = c / CH, ch = c % CH;
        const bool ok = r < nvalid;
        const long long row = ((base + (ok ? r : 0)) * nkv + kvh) * HD + ch * 8;
        cp_async16(smem_u32(Ks + swz<CH>(r, ch) * 8), kc + row, ok ? 16 : 0);
        cp_async16(smem_u32(Vs + swz<CH>(r, ch) * 8), vc + row, ok ? 16 : 0);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < ST - 1; ++k) issue(k);
  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  float mrow = -INFINITY, lrow = 0.f;
  for (int k = 0; k < n_my; ++k) {
    issue(k + ST - 1);
    cp_async_wait<ST - 1>();
    __syncwarp();
    const int t0 = t_begin + (w + k * W) * BT;
    const int nvalid = min(BT, t_end - t0);
    const bf16* Ks = ring + (k % ST) * 2 * TILE;
    const bf16* Vs = Ks + TILE;
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      uint32_t bfr[4];
      ldsm_x4(bfr, smem_u32(Ks + swz<CH>(((lane >> 4) << 3) + (lane & 7), 2 * kk + ((lane >> 3) & 1)) * 8));
      mma16816(s[0], qf[kk], bfr[0], bfr[1]);
      mma16816(s[1], qf[kk], bfr[2], bfr[3]);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = 8 * j + 2 * t + e;
        const float v = key < nvalid ? s[j][e] * scale_log2 : -INFINITY;
        s[j][e] = v;
        mx = fmaxf(mx, v);
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mnew = fmaxf(mrow, mx);
    const float muse = mnew == -INFINITY ? 0.f : mnew;
    const float alpha = exp2f(mrow - muse);
    mrow = mnew;
    lrow *= alpha;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      oacc[j][0] *= alpha;
      oacc[j][1] *= alpha;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      s[j][0] = exp2f(s[j][0] - muse);
      s[j][1] = exp2f(s[j][1] - muse);
      lrow += s[j][0] + s[j][1];
    }
    uint32_t a[4];
    a[0] = pack_bf16(s[0][0], s[0][1]);
    a[1] = 0u;
    a[2] = pack_bf16(s[1][0], s[1][1]);
    a[3] = 0u;
#pragma unroll
    for (int dp = 0; dp < NT / 2; ++dp) {
      uint32_t bfr[4];
      ldsm_x4_t(bfr, smem_u32(Vs + swz<CH>(lane & 15, 2 * dp + (lane >> 4)) * 8));
      mma16816(oacc[2 * dp], a, bfr[0], bfr[1]);
      mma16816(oacc[2 * dp + 1], a, bfr[2], bfr[3]);
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  lrow += __shfl_xor_sync(0xffffffffu, lrow, 1);
  lrow += __shfl_xor_sync(0xffffffffu, lrow, 2);
  __syncthreads();  // every warp is done with its ring: reuse it for the merge
  constexpr int RS = HD + 2;
  float* red = reinterpret_cast<float*>(smem_raw);  // [W][G][HD+2]
  if (g < G) {
    float* rw = red + ((size_t)w * G + g) * RS;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      rw[8 * j + 2 * t] = oacc[j][0];
      rw[8 * j + 2 * t + 1] = oacc[j][1];
    }
    if (t == 0) {
      rw[HD] = mrow;
      rw[HD + 1] = lrow;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * HD; e += W * 32) {
    const int gg = e / HD, d = e % HD;
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < W; ++k) M = fmaxf(M, red[((size_t)k * G + gg) * RS + HD]);
    float Lsum = 0.f, O = 0.f;
#pragma unroll
    for (int k = 0; k < W; ++k) {
      const float* rk = red + ((size_t)k * G + gg) * RS;
      const float f = rk[HD] == -INFINITY ? 0.f : exp2f(rk[HD] - M);
      Lsum += rk[HD + 1] * f;
      O += rk[d] * f;
    }
    const int h = kvh * G + gg;
    if (part_o == nullptr) {
      out[(long long)b * nq * HD + h * HD + d] = __float2bfloat16_rn(Lsum > 0.f ? O / Lsum : 0.f);
    } else {
      const long long pi = ((long long)(b * nq + h) * gridDim.z + split);
      part_o[pi * HD + d] = O;
      if (d == 0) {
        part_ml[pi * 2] = M;
        part_ml[pi * 2 + 1] = Lsum;
      }
    }
  }
}

template <int HD>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int splits,
                                      int nq, bf16* __restrict__ out) {
  pdl_launch_dependents();
  const int bh = blockIdx.x;  // b * nq + h
  const int d = threadIdx.x;
  if (d >= HD) return;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[((long long)bh * splits + s) * 2]);
  float Lsum = 0.f, O = 0.f;
  for (int s = 0; s < splits; ++s) {
    const long long pi = (long long)bh * splits + s;
    const float ms = part_ml[pi * 2];
    const float f = ms == -INFINITY ? 0.f : exp2f(ms - M);
    Lsum += part_ml[pi * 2 + 1] * f;
    O += part_o[pi * HD + d] * f;
  }
  out[(long long)bh * HD + d] = __float2bfloat16_rn(Lsum > 0.f ? O / Lsum : 0.f);
}

// ============================================================ flash forward
template <int HD>
__global__ void __launch_bounds__(128)
fa_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, long long qs,
              long long ks, long long vs, const int* __restrict__ cu, int nq, int nkv, float scale_log2, int causal,
              bf16* __restrict__ o, float* __restrict__ lse, int T_total, const int* __restrict__ seg,
              const uint32_t* __restrict__ cp_flags, uint32_t cp_epoch, int cp_size, long long wait_cycles) {
  constexpr int BM = 64, BN = 64, CH = HD / 8, KS = HD / 16, NT = HD / 8;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* Qs = reinterpret_cast<bf16*>(smem_raw);
  bf16* Ks = Qs + BM * HD;
  bf16* Vs = Ks + 2 * BN * HD;
  const int h = blockIdx.x;
  const int mblk = gridDim.y - 1 - blockIdx.y;
  const int b = blockIdx.z;
  // segment b: queries [s0, s0 + L), keys [k0, k0 + Lk); causal is bottom-right
  // aligned (query i sees keys <= i + off), which is the plain causal mask when
  // the two ranges coincide (seg == nullptr: packed varlen attention)
  const int s0 = seg ? seg[4 * b] : cu[b];
  const int L = seg ? seg[4 * b + 1] : cu[b + 1] - s0;
  const int k0 = seg ? seg[4 * b + 2] : s0;
  const int Lk = seg ? seg[4 * b + 3] : L;
  const int off = Lk - L;
  const int m0 = mblk * BM;
  if (m0 >= L) return;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int kvh = h / (nq / nkv);
  const bf16* qg = q + (long long)(s0 + m0) * qs + (long long)h * HD;
  const bf16* kg = k + (long long)k0 * ks + (long long)kvh * HD;
  const bf16* vg = v + (long long)k0 * vs + (long long)kvh * HD;
  load_tile<CH>(Qs, qg, qs, BM, min(BM, L - m0), tid, 128);
  const int n_end = causal ? min(Lk, m0 + BM + off) : Lk;
  const int nblocks = (n_end + BN - 1) / BN;
  // context parallelism with the K/V exchange in flight: key block n0 belongs to
  // chunk n0 / chunk_len of its sequence, owned by rank c (c < cp) or 2cp-1-c;
  // its rows are valid once that rank's copy flag reaches the epoch
  auto wait_keys = [&](int n0) {
    if (cp_flags != nullptr) {
      if (tid == 0) {
        const int c = n0 / L;  // every chunk has the segment's query length
        const int owner = c < cp_size ? c : 2 * cp_size - 1 - c;
        if (!cp_wait_flag(cp_flags + owner, cp_epoch, wait_cycles)) atomicExch(&g_attn_error, 1);
      }
      __syncthreads();
    }
  };
  wait_keys(0);
  load_tile<CH>(Ks, kg, ks, BN, min(BN, Lk), tid, 128);
  load_tile<CH>(Vs, vg, vs, BN, min(BN, Lk), tid, 128);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  uint32_t qf[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) ldsm_x4(qf[kk], smem_u32(Qs + swz<CH>(16 * w + (lane & 15), 2 * kk + (lane >> 4)) * 8));

  float oacc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int qrow0 = m0 + 16 * w + g;

  for (int nb = 0; nb < nblocks; ++nb) {
    const int buf = nb & 1;
    if (nb + 1 < nblocks) {
      const int n1 = (nb + 1) * BN;
      wait_keys(n1);
      load_tile<CH>(Ks + (buf ^ 1) * BN * HD, kg + (long long)n1 * ks, ks, BN, min(BN, Lk - n1), tid, 128);
      load_tile<CH>(Vs + (buf ^ 1) * BN * HD, vg + (long long)n1 * vs, vs, BN, min(BN, Lk - n1), tid, 128);
      cp_async_commit();
    }
    const bf16* Kb = Ks + buf * BN * HD;
    const bf16* Vb = Vs + buf * BN * HD;
    float sacc[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t bfr[4];
        ldsm_x4(bfr, smem_u32(Kb + swz<CH>(np * 16 + ((lane >> 4) << 3) + (lane & 7), 2 * kk + ((lane >> 3) & 1)) * 8));
        mma16816(sacc[2 * np], qf[kk], bfr[0], bfr[1]);
        mma16816(sacc[2 * np + 1], qf[kk], bfr[2], bfr[3]);
      }
    }
    const int n0 = nb * BN;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = n0 + 8 * j + 2 * t + (e & 1);
        const int qr = qrow0 + ((e >> 1) << 3);
        float sv = sacc[j][e] * scale_log2;
        if (key >= Lk || (causal && key > qr + off)) sv = -INFINITY;
        sacc[j][e] = sv;
        mx[e >> 1] = fmaxf(mx[e >> 1], sv);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(mrow[r], mx[r]);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      const float alpha = exp2f(mrow[r] - muse);
      mrow[r] = mnew;
      lrow[r] *= alpha;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        oacc[j][2 * r] *= alpha;
        oacc[j][2 * r + 1] *= alpha;
      }
      mx[r] = muse;
    }
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(sacc[j][e] - mx[e >> 1]);
        sacc[j][e] = p;
        lrow[e >> 1] += p;
      }
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(sacc[2 * kk][0], sacc[2 * kk][1]);
      a[1] = pack_bf16(sacc[2 * kk][2], sacc[2 * kk][3]);
      a[2] = pack_bf16(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      a[3] = pack_bf16(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < NT / 2; ++dp) {
        uint32_t bfr[4];
        ldsm_x4_t(bfr, smem_u32(Vb + swz<CH>(kk * 16 + (lane & 15), 2 * dp + (lane >> 4)) * 8));
        mma16816(oacc[2 * dp], a, bfr[0], bfr[1]);
        mma16816(oacc[2 * dp + 1], a, bfr[2], bfr[3]);
      }
    }
    cp_async_wait_all();
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qr = qrow0 + 8 * r;
    if (qr >= L) continue;
    const float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    bf16* orow = o + ((long long)(s0 + qr) * nq + h) * HD;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      *reinterpret_cast<__nv_bfloat162*>(orow + 8 * j + 2 * t) =
          __floats2bfloat162_rn(oacc[j][2 * r] * inv, oacc[j][2 * r + 1] * inv);
    }
    if (t == 0) lse[(long long)h * T_total + s0 + qr] = mrow[r] * 0.69314718055994531f + logf(lrow[r]);
  }
}

// ============================================================ flash backward
template <int HD>
__global__ void fa_bwd_pre_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ out, int rows,
                                  float* __restrict__ D, int nq, int T_total) {
  const int lane = threadIdx.x & 31;
  const long long r = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5);  // token * nq + h
  if (r >= rows) return;
  float s = 0.f;
  for (int d = lane; d < HD; d += 32) s += __bfloat162float(dout[r * HD + d]) * __bfloat162float(out[r * HD + d]);
  s = warp_sum(s);
  if (lane == 0) {
    const long long tok = r / nq;
    const int h = r % nq;
    D[(long long)h * T_total + tok] = s;
  }
}

template <int HD>
__global__ void __launch_bounds__(128)
fa_bwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, long long qs,
              long long ks, long long vs, const bf16* __restrict__ dout, const float* __restrict__ lse,
              const float* __restrict__ Dv, const int* __restrict__ cu, int nq, int nkv, float scale,
              float scale_log2, int causal, float* __restrict__ dq_acc, bf16* __restrict__ dk, bf16* __restrict__ dv,
              int T_total, const int* __restrict__ seg, float* __restrict__ dk_acc, float* __restrict__ dv_acc) {
  constexpr int BN = 64, BM = 32, CH = HD / 8, KS = HD / 16, NT = HD / 8;
  constexpr int QCH = BM / 8;  // chunks per dS^T row
  extern __shared__ __align__(128) unsigned char smem_raw[];
  bf16* Ks = reinterpret_cast<bf16*>(smem_raw);
  bf16* Vs = Ks + BN * HD;
  bf16* Qs = Vs + BN * HD;
  bf16* dOs = Qs + BM * HD;
  bf16* dSs = dOs + BM * HD;
  float* lse_s = reinterpret_cast<float*>(dSs + BN * BM);
  float* D_s = lse_s + BM;
  const int kvh = blockIdx.x, nblk = blockIdx.y, b = blockIdx.z;
  // segment b (see fa_fwd_kernel): queries [s0, s0 + L), keys [k0, k0 + Lk)
  const int s0 = seg ? seg[4 * b] : cu[b];
  const int L = seg ? seg[4 * b + 1] : cu[b + 1] - s0;
  const int k0 = seg ? seg[4 * b + 2] : s0;
  const int Lk = seg ? seg[4 * b + 3] : L;
  const int off = Lk - L;
  const int n0 = nblk * BN;
  if (n0 >= Lk) return;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int G = nq / nkv;
  const float log2e = 1.4426950408889634f;
  load_tile<CH>(Ks, k + (long long)(k0 + n0) * ks + (long long)kvh * HD, ks, BN, min(BN, Lk - n0), tid, 128);
  load_tile<CH>(Vs, v + (long long)(k0 + n0) * vs + (long long)kvh * HD, vs, BN, min(BN, Lk - n0), tid, 128);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  float dka[NT][4], dva[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) dka[j][e] = dva[j][e] = 0.f;

  const int m_begin = causal ? (max(0, n0 - off) / BM) * BM : 0;
  const int key0 = n0 + 16 * w + g;  // this thread's key rows: key0, key0 + 8
  for (int hq = 0; hq < G; ++hq) {
    const int h = kvh * G + hq;
    for (int m0 = m_begin; m0 < L; m0 += BM) {
      load_tile<CH>(Qs, q + (long long)(s0 + m0) * qs + (long long)h * HD, qs, BM, min(BM, L - m0), tid, 128);
      load_tile<CH>(dOs, dout + ((long long)(s0 + m0) * nq + h) * HD, (long long)nq * HD, BM, min(BM, L - m0), tid,
                    128);
      cp_async_commit();
      if (tid < BM) {
        const int qq = m0 + tid;
        lse_s[tid] = qq < L ? lse[(long long)h * T_total + s0 + qq] * log2e : INFINITY;
        D_s[tid] = qq < L ? Dv[(long long)h * T_total + s0 + qq] : 0.f;
      }
      cp_async_wait_all();
      __syncthreads();
      // S^T = K_w Q^T  -> [16 keys x 32 queries] = 4 n-tiles
      float st[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, smem_u32(Ks + swz<CH>(16 * w + (lane & 15), 2 * kk + (lane >> 4)) * 8));
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bfr[4];
          ldsm_x4(bfr, smem_u32(Qs + swz<CH>(np * 16 + ((lane >> 4) << 3) + (lane & 7), 2 * kk + ((lane >> 3) & 1)) * 8));
          mma16816(st[2 * np], a, bfr[0], bfr[1]);
          mma16816(st[2 * np + 1], a, bfr[2], bfr[3]);
        }
      }
      // P^T
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = key0 + ((e >> 1) << 3);
          const int ql = 8 * j + 2 * t + (e & 1);
          const int qq = m0 + ql;
          const bool ok = qq < L && key < Lk && (!causal || key <= qq + off);
          st[j][e] = ok ? exp2f(st[j][e] * scale_log2 - lse_s[ql]) : 0.f;
        }
      }
      // dV += P^T dO
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
        a[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
        a[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
        a[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < NT / 2; ++dp) {
          uint32_t bfr[4];
          ldsm_x4_t(bfr, smem_u32(dOs + swz<CH>(kk * 16 + (lane & 15), 2 * dp + (lane >> 4)) * 8));
          mma16816(dva[2 * dp], a, bfr[0], bfr[1]);
          mma16816(dva[2 * dp + 1], a, bfr[2], bfr[3]);
        }
      }
      // dP^T = V_w dO^T
      float dpt[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) dpt[j][0] = dpt[j][1] = dpt[j][2] = dpt[j][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t a[4];
        ldsm_x4(a, smem_u32(Vs + swz<CH>(16 * w + (lane & 15), 2 * kk + (lane >> 4)) * 8));
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t bfr[4];
          ldsm_x4(bfr, smem_u32(dOs + swz<CH>(np * 16 + ((lane >> 4) << 3) + (lane & 7), 2 * kk + ((lane >> 3) & 1)) * 8));
          mma16816(dpt[2 * np], a, bfr[0], bfr[1]);
          mma16816(dpt[2 * np + 1], a, bfr[2], bfr[3]);
        }
      }
      // dS^T = P^T * (dP^T - D)
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[j][e] = st[j][e] * (dpt[j][e] - D_s[8 * j + 2 * t + (e & 1)]);
      // dK += dS^T Q
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
        a[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
        a[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
        a[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < NT / 2; ++dp) {
          uint32_t bfr[4];
          ldsm_x4_t(bfr, smem_u32(Qs + swz<CH>(kk * 16 + (lane & 15), 2 * dp + (lane >> 4)) * 8));
          mma16816(dka[2 * dp], a, bfr[0], bfr[1]);
          mma16816(dka[2 * dp + 1], a, bfr[2], bfr[3]);
        }
      }
      // stash dS^T [64 keys x 32 q] (bf16) for the dQ product
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = 16 * w + g + 8 * r;
          const int col = 8 * j + 2 * t;
          bf16* dst = dSs + swz<QCH>(row, col >> 3) * 8 + (col & 7);
          *reinterpret_cast<uint32_t*>(dst) = pack_bf16(st[j][2 * r], st[j][2 * r + 1]);
        }
      }
      __syncthreads();
      // dQ[32 q x HD] += dS[32 q x 64 keys] K[64 keys x HD]; warp w: m-tile (w & 1), n-tiles [(w>>1)*NT/2, +NT/2)
      {
        const int mt = w & 1;
        const int nt0 = (w >> 1) * (NT / 2);
        float dqa[NT / 2][4];
#pragma unroll
        for (int j = 0; j < NT / 2; ++j) dqa[j][0] = dqa[j][1] = dqa[j][2] = dqa[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          uint32_t a[4];
          const int key = 16 * kk + (lane & 7) + ((lane >> 4) << 3);
          const int qch = 2 * mt + ((lane >> 3) & 1);
          ldsm_x4_t(a, smem_u32(dSs + swz<QCH>(key, qch) * 8));
#pragma unroll
          for (int j = 0; j < NT / 2; ++j) {
            uint32_t bfr[2];
            ldsm_x2_t(bfr, smem_u32(Ks + swz<CH>(16 * kk + (lane & 15), nt0 + j) * 8));
            mma16816(dqa[j], a, bfr[0], bfr[1]);
          }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int qq = m0 + 16 * mt + g + 8 * r;
          if (qq >= L) continue;
          float* dst = dq_acc + ((long long)(s0 + qq) * nq + h) * HD;
#pragma unroll
          for (int j = 0; j < NT / 2; ++j) {
            atomicAdd(reinterpret_cast<float2*>(dst + 8 * (nt0 + j) + 2 * t), make_float2(dqa[j][2 * r], dqa[j][2 * r + 1]));
          }
        }
      }
      __syncthreads();
    }
  }
  // epilogue: dK (scaled), dV
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = key0 + 8 * r;
    if (key >= Lk) continue;
    if (dk_acc != nullptr) {
      // segments may share keys (context-parallel chunks of one sequence): accumulate
      float* dka_r = dk_acc + ((long long)(k0 + key) * nkv + kvh) * HD;
      float* dva_r = dv_acc + ((long long)(k0 + key) * nkv + kvh) * HD;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        atomicAdd(reinterpret_cast<float2*>(dka_r + 8 * j + 2 * t), make_float2(dka[j][2 * r], dka[j][2 * r + 1]));
        atomicAdd(reinterpret_cast<float2*>(dva_r + 8 * j + 2 * t), make_float2(dva[j][2 * r], dva[j][2 * r + 1]));
      }
      continue;
    }
    bf16* dkr = dk + ((long long)(k0 + key) * nkv + kvh) * HD;
    bf16* dvr = dv + ((long long)(k0 + key) * nkv + kvh) * HD;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      *reinterpret_cast<__nv_bfloat162*>(dkr + 8 * j + 2 * t) =
          __floats2bfloat162_rn(dka[j][2 * r] * scale, dka[j][2 * r + 1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(dvr + 8 * j + 2 * t) = __floats2bfloat162_rn(dva[j][2 * r], dva[j][2 * r + 1]);
    }
  }
}

__global__ void dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, long long n, float scale) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dq[i] = __float2bfloat16_rn(acc[i] * scale);
}

}  // namespace rlb

using namespace rlb;

#define RLB_HD_SWITCH(HDV, ...)                          \
  [&] {                                                  \
    if ((HDV) == 128) {                                  \
      constexpr int HD = 128;                            \
      return __VA_ARGS__();                              \
    } else if ((HDV) == 64) {                            \
      constexpr int HD = 64;                             \
      return __VA_ARGS__();                              \
    } else if ((HDV) == 32) {                            \
      constexpr int HD = 32;                             \
      return __VA_ARGS__();                              \
    } else if ((HDV) == 16) {                            \
      constexpr int HD = 16;                             \
      return __VA_ARGS__();                              \
    } else {                                             \
      TORCH_CHECK(false, "rl_b200: head_dim ", HDV, " unsupported (16/32/64/128)"); \
    }                                                    \
  }()

static void check_head_view(const at::Tensor& x, const char* name) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3 && x.scalar_type() == at::kBFloat16, "rl_b200 attention: ", name,
              " must be a bf16 CUDA [T, heads, hd] tensor");
  TORCH_CHECK(x.stride(2) == 1 && x.stride(1) == x.size(2), "rl_b200 attention: ", name,
              " must have contiguous heads within a token");
  TORCH_CHECK(x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "rl_b200 attention: ", name, " rows must be 16-byte aligned");
}

std::vector<at::Tensor> flash_attn_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cu_seqlens,
                                       int64_t max_seqlen, double scale, bool causal) {
  check_head_view(q, "q");
  check_head_view(k, "k");
  check_head_view(v, "v");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T_ = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k.size(1);
  TORCH_CHECK(nq % nkv == 0, "rl_b200 attention: nq must be a multiple of nkv");
  auto cu = cu_seqlens.to(at::kInt).contiguous();
  const int B = cu.size(0) - 1;
  auto o = at::empty({T_, nq, hd}, q.options());
  auto lse = at::empty({nq, T_}, q.options().dtype(at::kFloat));
  if (T_ == 0 || B == 0 || max_seqlen == 0) return {o, lse};
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  RLB_HD_SWITCH(hd, [&] {
    const int smem = (64 * HD + 2 * 64 * HD * 2) * 2;
    auto kern = fa_fwd_kernel<HD>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(nq, (max_seqlen + 63) / 64, B);
    kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(),
                                        q.stride(0), k.stride(0), v.stride(0), cu.data_ptr<int>(), nq, nkv, scale_log2,
                                        causal ? 1 : 0, (bf16*)o.data_ptr(), lse.data_ptr<float>(), T_, nullptr,
                                        nullptr, 0u, 0, (long long)peer_wait_cycles());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {o, lse};
}

std::vector<at::Tensor> flash_attn_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                                       at::Tensor lse, at::Tensor cu_seqlens, int64_t max_seqlen, double scale,
                                       bool causal) {
  check_head_view(q, "q");
  check_head_view(k, "k");
  check_head_view(v, "v");
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous(), "rl_b200 attention bwd: dout/out must be contiguous");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T_ = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k.size(1);
  auto cu = cu_seqlens.to(at::kInt).contiguous();
  const int B = cu.size(0) - 1;
  auto dq = at::empty({T_, nq, hd}, q.options());
  auto dk = at::zeros({T_, nkv, hd}, q.options());
  auto dv = at::zeros({T_, nkv, hd}, q.options());
  if (T_ == 0 || B == 0) return {dq, dk, dv};
  auto D = at::empty({nq, T_}, q.options().dtype(at::kFloat));
  auto dq_acc = at::zeros({T_, nq, hd}, q.options().dtype(at::kFloat));
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  RLB_HD_SWITCH(hd, [&] {
    const int rows = T_ * nq;
    fa_bwd_pre_kernel<HD><<<(rows + 7) / 8, 256, 0, stream()>>>((const bf16*)dout.data_ptr(), (const bf16*)out.data_ptr(),
                                                                 rows, D.data_ptr<float>(), nq, T_);
    const int smem = (64 * HD * 2 + 32 * HD * 2 + 64 * 32) * 2 + 2 * 32 * 4;
    auto kern = fa_bwd_kernel<HD>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(nkv, (max_seqlen + 63) / 64, B);
    kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(),
                                        q.stride(0), k.stride(0), v.stride(0), (const bf16*)dout.data_ptr(),
                                        lse.data_ptr<float>(), D.data_ptr<float>(), cu.data_ptr<int>(), nq, nkv,
                                        (float)scale, scale_log2, causal ? 1 : 0, dq_acc.data_ptr<float>(),
                                        (bf16*)dk.data_ptr(), (bf16*)dv.data_ptr(), T_, nullptr, nullptr, nullptr);
  });
  const long long n = (long long)T_ * nq * hd;
  dq_convert_kernel<<<(int)std::min<long long>((n + 255) / 256, (long long)num_sms() * 8), 256, 0, stream()>>>(
      dq_acc.data_ptr<float>(), (bf16*)dq.data_ptr(), n, (float)scale);
  RLB_CUDA_CHECK(cudaGetLastError());
  return {dq, dk, dv};
}

// Segment attention (context parallelism): segment b attends queries
// [seg[b][0], +seg[b][1]) of q to keys [seg[b][2], +seg[b][3]) of k / v, causal
// with the last query aligned to the last key.  Segments may share keys.
// With cp_flags (int32 [cp] on the device) the kernel waits, per key block, for
// the flag of the rank owning that block's chunk to reach cp_epoch: the K/V
// exchange of context parallelism may still be landing (copy engines) when the
// kernel starts.  Chunk lengths must be multiples of 64 (one key block).
std::vector<at::Tensor> flash_attn_seg_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor seg, int64_t max_q,
                                           double scale, c10::optional<at::Tensor> cp_flags, int64_t cp_epoch,
                                           int64_t cp_size) {
  check_head_view(q, "q");
  check_head_view(k, "k");
  check_head_view(v, "v");
  TORCH_CHECK(seg.is_cuda() && seg.scalar_type() == at::kInt && seg.dim() == 2 && seg.size(1) == 4 &&
              seg.is_contiguous(), "rl_b200 segment attention: seg int32 [S, 4]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T_ = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k.size(1);
  TORCH_CHECK(nq % nkv == 0, "rl_b200 attention: nq must be a multiple of nkv");
  const int S = seg.size(0);
  auto o = at::zeros({T_, nq, hd}, q.options());
  auto lse = at::zeros({nq, T_}, q.options().dtype(at::kFloat));
  if (T_ == 0 || S == 0 || max_q == 0) return {o, lse};
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  RLB_HD_SWITCH(hd, [&] {
    const int smem = (64 * HD + 2 * 64 * HD * 2) * 2;
    auto kern = fa_fwd_kernel<HD>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(nq, (max_q + 63) / 64, S);
    kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(),
                                        q.stride(0), k.stride(0), v.stride(0), nullptr, nq, nkv, scale_log2, 1,
                                        (bf16*)o.data_ptr(), lse.data_ptr<float>(), T_, seg.data_ptr<int>(),
                                        cp_flags ? reinterpret_cast<const uint32_t*>(cp_flags->data_ptr<int>())
                                                 : nullptr,
                                        (uint32_t)cp_epoch, (int)cp_size, (long long)peer_wait_cycles());
  });
  RLB_CUDA_CHECK(cudaGetLastError());
  return {o, lse};
}

std::vector<at::Tensor> flash_attn_seg_bwd(at::Tensor dout, at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor out,
                                           at::Tensor lse, at::Tensor seg, int64_t max_k, double scale) {
  check_head_view(q, "q");
  check_head_view(k, "k");
  check_head_view(v, "v");
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous(), "rl_b200 attention bwd: dout/out must be contiguous");
  TORCH_CHECK(seg.is_cuda() && seg.scalar_type() == at::kInt && seg.dim() == 2 && seg.size(1) == 4 &&
              seg.is_contiguous(), "rl_b200 segment attention: seg int32 [S, 4]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T_ = q.size(0), nq = q.size(1), hd = q.size(2), nkv = k.size(1), Tk = k.size(0);
  const int S = seg.size(0);
  auto dq = at::zeros({T_, nq, hd}, q.options());
  auto dk_acc = at::zeros({Tk, nkv, hd}, q.options().dtype(at::kFloat));
  auto dv_acc = at::zeros({Tk, nkv, hd}, q.options().dtype(at::kFloat));
  if (T_ == 0 || S == 0) return {dq, dk_acc.to(q.scalar_type()), dv_acc.to(q.scalar_type())};
  auto D = at::empty({nq, T_}, q.options().dtype(at::kFloat));
  auto dq_acc = at::zeros({T_, nq, hd}, q.options().dtype(at::kFloat));
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  RLB_HD_SWITCH(hd, [&] {
    const int rows = T_ * nq;
    fa_bwd_pre_kernel<HD><<<(rows + 7) / 8, 256, 0, stream()>>>((const bf16*)dout.data_ptr(), (const bf16*)out.data_ptr(),
                                                                 rows, D.data_ptr<float>(), nq, T_);
    const int smem = (64 * HD * 2 + 32 * HD * 2 + 64 * 32) * 2 + 2 * 32 * 4;
    auto kern = fa_bwd_kernel<HD>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    dim3 grid(nkv, (max_k + 63) / 64, S);
    kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), (const bf16*)v.data_ptr(),
                                        q.stride(0), k.stride(0), v.stride(0), (const bf16*)dout.data_ptr(),
                                        lse.data_ptr<float>(), D.data_ptr<float>(), nullptr, nq, nkv, (float)scale,
                                        scale_log2, 1, dq_acc.data_ptr<float>(), nullptr, nullptr, T_,
                                        seg.data_ptr<int>(), dk_acc.data_ptr<float>(), dv_acc.data_ptr<float>());
  });
  const long long n = (long long)T_ * nq * hd;
  dq_convert_kernel<<<(int)std::min<long long>((n + 255) / 256, (long long)num_sms() * 8), 256, 0, stream()>>>(
      dq_acc.data_ptr<float>(), (bf16*)dq.data_ptr(), n, (float)scale);
  RLB_CUDA_CHECK(cudaGetLastError());
  return {dq, dk_acc.mul(scale).to(q.scalar_type()), dv_acc.to(q.scalar_type())};
}

at::Tensor paged_decode_attn(at::Tensor q, at::Tensor k_cache, at::Tensor v_cache, at::Tensor block_tables,
                             at::Tensor seq_lens, double scale, int64_t max_seq_len, double k_scale, double v_scale) {
  TORCH_CHECK(q.is_cuda() && q.dim() == 3 && q.scalar_type() == at::kBFloat16, "decode: q must be bf16 [B, nq, hd]");
  TORCH_CHECK(q.stride(2) == 1 && q.stride(1) == q.size(2), "decode: q heads must be contiguous");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4, "decode: caches [nb, bs, nkv, hd]");
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = q.size(0), nq = q.size(1), hd = q.size(2);
  const int bs = k_cache.size(1), nkv = k_cache.size(2);
  TORCH_CHECK(k_cache.size(3) == hd && nq % nkv == 0, "decode: shape mismatch");
  const int G = nq / nkv;
  auto bt = block_tables.to(at::kInt).contiguous();
  auto sl = seq_lens.to(at::kInt).contiguous();
  auto out = at::empty({B, nq, hd}, q.options());
  if (B == 0) return out;
  const int max_blocks = bt.size(1);
  const int cap = max_seq_len > 0 ? (int)max_seq_len : max_blocks * bs;
  const bool fp8 = k_cache.scalar_type() == at::kFloat8_e4m3fn;
  // pipelined tensor-core kernel: W=4 warps x ST=3 stages x 16-token tiles,
  // two CTAs per SM; the split count makes the grid a near-whole number of
  // waves of those 2 x SMs slots
  constexpr int kW = 4, kST = 3;
  const bool pipe = !fp8 && hd >= 64 && bs % 16 == 0;
  int splits = 1;
  const int base_ctas = B * nkv;
  if (pipe) {
    const int slots = 2 * num_sms();
    const int max_s = std::max(1, std::min(8, cap / 128));
    double best = -1.0;
    for (int s_ = 1; s_ <= max_s; ++s_) {
      const double waves = (double)base_ctas * s_ / slots;
      const double eff = waves / std::ceil(waves);
      if (eff > best + 0.02) {
        best = eff;
        splits = s_;
      }
      if (eff >= 0.95) break;
    }
  } else {
    const int target = 2 * num_sms();
    if (base_ctas < target) splits = std::min((target + base_ctas - 1) / base_ctas, std::max(1, cap / 256));
  }
  const int tps = ((cap + splits - 1) / splits + 127) / 128 * 128;
  splits = (cap + tps - 1) / tps;
  at::Tensor part_o, part_ml;
  if (splits > 1) {
    part_o = at::empty({(long long)B * nq * splits, hd}, q.options().dtype(at::kFloat));
    part_ml = at::empty({(long long)B * nq * splits, 2}, q.options().dtype(at::kFloat));
  }
  const float scale_log2 = (float)(scale * 1.4426950408889634);
  auto launch = [&](auto gtag, auto ctag) {
    constexpr int GG = decltype(gtag)::value;
    using C = typename decltype(ctag)::type;
    RLB_HD_SWITCH(hd, [&] {
      if constexpr (HD >= 64 && std::is_same<C, bf16>::value) {
        dim3 grid(B, nkv, splits);
        if (pipe) {
          const int ring = kW * kST * 2 * 16 * HD * 2;
          const int nbt = tps / bs + 2;
          const int smem = std::max(ring + nbt * 4, kW * GG * (HD + 2) * 4 + nbt * 4);
          TORCH_CHECK(smem <= 227 * 1024, "decode: block table of a split does not fit in shared memory");
          auto kern = paged_decode_pipe_kernel<HD, GG, kW, kST>;
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
          kern<<<grid, kW * 32, smem, stream()>>>(
              (const bf16*)q.data_ptr(), q.stride(0), (const bf16*)k_cache.data_ptr(),
              (const bf16*)v_cache.data_ptr(), bt.data_ptr<int>(), max_blocks, sl.data_ptr<int>(), bs, nkv,
              scale_log2, tps, splits > 1 ? part_o.data_ptr<float>() : nullptr,
              splits > 1 ? part_ml.data_ptr<float>() : nullptr, (bf16*)out.data_ptr(), (int)k_cache.size(0));
          RLB_CUDA_CHECK(cudaGetLastError());
          if (splits > 1)
            decode_combine_kernel<HD><<<B * nq, HD, 0, stream()>>>(
                part_o.data_ptr<float>(), part_ml.data_ptr<float>(), splits, nq, (bf16*)out.data_ptr());
          return;
        }
        const int smem = 4 * 2 * 32 * HD * 2 + 4 * GG * (HD + 2) * 4;
        auto kern = paged_decode_tc_kernel<HD, GG>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        kern<<<grid, 128, smem, stream()>>>(
            (const bf16*)q.data_ptr(), q.stride(0), (const bf16*)k_cache.data_ptr(), (const bf16*)v_cache.data_ptr(),
            bt.data_ptr<int>(), max_blocks, sl.data_ptr<int>(), bs, nkv, scale_log2, tps,
            splits > 1 ? part_o.data_ptr<float>() : nullptr, splits > 1 ? part_ml.data_ptr<float>() : nullptr,
            (bf16*)out.data_ptr());
        if (splits > 1)
          decode_combine_kernel<HD><<<B * nq, HD, 0, stream()>>>(part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                                                 splits, nq, (bf16*)out.data_ptr());
      } else if constexpr (HD >= 32) {
        dim3 grid(B, nkv, splits);
        paged_decode_kernel<C, HD, GG><<<grid, 128, 0, stream()>>>(
            (const bf16*)q.data_ptr(), q.stride(0), (const C*)k_cache.data_ptr(), (const C*)v_cache.data_ptr(),
            bt.data_ptr<int>(), max_blocks, sl.data_ptr<int>(), bs, nkv, scale_log2, (float)k_scale, (float)v_scale,
            tps, splits > 1 ? part_o.data_ptr<float>() : nullptr, splits > 1 ? part_ml.data_ptr<float>() : nullptr,
            (bf16*)out.data_ptr());
        if (splits > 1)
          decode_combine_kernel<HD><<<B * nq, HD, 0, stream()>>>(part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                                                 splits, nq, (bf16*)out.data_ptr());
      } else {
        TORCH_CHECK(false, "decode attention needs head_dim >= 32");
      }
    });
  };
  struct BF { using type = bf16; };
  struct F8 { using type = __nv_fp8_e4m3; };
  TORCH_CHECK(fp8 || k_cache.scalar_type() == at::kBFloat16, "decode: cache must be bf16 or fp8 e4m3");
  auto dispatch_c = [&](auto gtag) {
    if (fp8) launch(gtag, F8{}); else launch(gtag, BF{});
  };
  switch (G) {
    case 1: dispatch_c(std::integral_constant<int, 1>{}); break;
    case 2: dispatch_c(std::integral_constant<int, 2>{}); break;
    case 4: dispatch_c(std::integral_constant<int, 4>{}); break;
    case 8: dispatch_c(std::integral_constant<int, 8>{}); break;
    default: TORCH_CHECK(false, "decode: GQA group size ", G, " unsupported (1/2/4/8)");
  }
  RLB_CUDA_CHECK(cudaGetLastError());
  return out;
}

int64_t attn_error_flag(bool reset) {
  int v = 0;
  RLB_CUDA_CHECK(cudaMemcpyFromSymbol(&v, rlb::g_attn_error, sizeof(int)));
  if (reset) {
    const int z = 0;
    RLB_CUDA_CHECK(cudaMemcpyToSymbol(rlb::g_attn_error, &z, sizeof(int)));
  }
  return v;
}

int64_t bounds_error_attention(bool reset) { return rlb::rlb_bounds_error(reset); }
