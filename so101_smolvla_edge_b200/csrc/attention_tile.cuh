// mma.sync flash attention, shared by the standalone attention kernel and the persistent expert
// step kernel.
//
// Grouped-query flash attention for SigLIP (1024 tokens, no mask), the SmolLM2 prefix (prefix-LM
// mask) and the action expert (self: prefix keys + causal own rows; cross: the expert's projections
// of the prefix keys). One CTA = 64 query rows of one head (4 warps x 16 rows); K/V stream through
// a double-buffered shared-memory ring of 64-key tiles (cp.async); S = Q K^T and O += P V on
// mma.sync m16n8k16 bf16 with fp32 accumulators; softmax online in fp32 with exp2; P rounded to bf16
// for PV, row sums from the fp32 P.
//
// Mask: key j is visible to query i iff j < Lk && (j < causal_from || j <= i + q_offset). Query
// head h reads kv head h / (nq / nkv). RoPE rotates q as it is staged (per-operation rounding,
// then one rounding to bf16).
#pragma once

#include "common.cuh"

namespace so101 {

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  void* o;
  long long ldq, ldk, ldv, ldo;
  long long bq, bk, bv, bo;
  int o_type;
  float o_qscale;
  int Lq, Lk, nq, nkv;
  long long causal_from, q_offset;
  const float* cos;
  const float* sin;
  float scale_log2;
  int kv_splits;  // > 1: the key tiles are split over a cluster of this many CTAs
  // Keys j >= own_from read row j - own_from of k_own / v_own (the step's own rows, straight from
  // the fused qkv output, batch stride b_own) instead of k / v; those keys are rotated by
  // k_cos / k_sin (row j - own_from) once they are in shared memory. k_own == nullptr: off.
  const __nv_bfloat16* k_own = nullptr;
  const __nv_bfloat16* v_own = nullptr;
  long long ld_own = 0, b_own = 0, own_from = 0;
  const float* k_cos = nullptr;
  const float* k_sin = nullptr;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Shared-memory bytes attention_body<HD, ..., NBUF> uses: the Q tile and NBUF K and V tiles.
template <int HD, int NBUF = 2>
constexpr int attention_smem_bytes() {
  return (1 + 2 * NBUF) * 64 * (HD + 8) * 2;
}

// One CTA's work (128 threads, all of which must call it): query rows [q0, q0 + 64) of head h of
// problem bi, key tiles of split `split` of a.kv_splits (SPLIT) or all of them. TILE_OUT (HD 64,
// no split): the normalised rows go to o_tile in shared memory instead of a.o, as bf16 in the
// K-major TMA SWIZZLE_128B layout (64 rows of 128 bytes; 16-byte chunk c of row r stored at chunk
// c ^ (r % 8); 1024-byte aligned), the B operand of a tcgen05 MMA; rows at or past Lq are zero.
// NBUF: depth of the K/V ring; NBUF - WG tiles are loaded ahead of the ones being used, so a CTA
// with at most NBUF - WG tiles (the expert's 291 keys at NBUF 6) pays one load latency in all.
// WG (TILE_OUT only): warp groups of 128 threads (the CTA has 128 * WG), which take the key tiles
// in turn, tile g + WG * i to group g, each with its own running max, sums and output rows; group 0
// merges the others' in group order at the end and writes the tile.
template <int HD, bool SPLIT, bool TILE_OUT = false, int NBUF = 2, int WG = 1>
__device__ __forceinline__ void attention_body(const AttnArgs& a, int split, int q0, int h, int bi,
                                               uint8_t* smem_raw, uint8_t* o_tile = nullptr) {
  static_assert(!TILE_OUT || (HD == 64 && !SPLIT), "the shared-memory output tile holds one 64-dim head");
  static_assert(WG == 1 || (TILE_OUT && NBUF >= 2 * WG), "warp groups: tile output, a ring of two rounds");
  constexpr int NT = 128 * WG;  // threads
  constexpr int BM = 64, BN = 64, LDS = HD + 8, HALF = HD / 2;
  constexpr int CHUNKS = HD / 8;  // 16-byte chunks per row
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  static_assert(NBUF >= 2, "the K/V ring needs two buffers");
  __nv_bfloat16* sK = sQ + BM * LDS;          // [NBUF][BN * LDS]
  __nv_bfloat16* sV = sK + NBUF * BN * LDS;   // [NBUF][BN * LDS]

  // warp: this thread's warp within its group (its 16 query rows); grp: its group
  const int tid = threadIdx.x, warp = (tid >> 5) & 3, lane = tid & 31, grp = tid >> 7;
  const int S = SPLIT ? a.kv_splits : 1;
  const int kvh = h / (a.nq / a.nkv);
  const __nv_bfloat16* Q = a.q + bi * a.bq + static_cast<long long>(h) * HD;
  const __nv_bfloat16* K = a.k + bi * a.bk + static_cast<long long>(kvh) * HD;
  const __nv_bfloat16* V = a.v + bi * a.bv + static_cast<long long>(kvh) * HD;
  const bool own = a.k_own != nullptr;
  const __nv_bfloat16* K_own = own ? a.k_own + bi * a.b_own + static_cast<long long>(kvh) * HD : nullptr;
  const __nv_bfloat16* V_own = own ? a.v_own + bi * a.b_own + static_cast<long long>(kvh) * HD : nullptr;

  // last key any query of this block can see -> number of key tiles
  long long last = a.causal_from - 1;
  const long long diag = static_cast<long long>(q0 + BM - 1) + a.q_offset;
  if (diag > last) last = diag;
  if (last > a.Lk - 1) last = a.Lk - 1;
  const int all_tiles = static_cast<int>((last + BN) / BN);
  const int per_split = (all_tiles + S - 1) / S;
  const int t_begin = split * per_split;
  const int t_end = min(all_tiles, t_begin + per_split);
  const int n_tiles = t_end > t_begin ? t_end - t_begin : 0;

  auto load_kv = [&](int tile, int buf) {
    const int j0 = tile * BN;
    for (int c = tid; c < BN * CHUNKS; c += NT) {
      const int r = c / CHUNKS, cc = c % CHUNKS;
      const int j = j0 + r;
      const bool ok = j < a.Lk;
      const long long jj = ok ? j : 0;
      const bool mine = own && jj >= a.own_from;
      const __nv_bfloat16* ks = mine ? K_own + (jj - a.own_from) * a.ld_own : K + jj * a.ldk;
      const __nv_bfloat16* vs = mine ? V_own + (jj - a.own_from) * a.ld_own : V + jj * a.ldv;
      cp_async16(smem_u32(sK + buf * BN * LDS + r * LDS + cc * 8), ks + cc * 8, ok ? 16 : 0);
      cp_async16(smem_u32(sV + buf * BN * LDS + r * LDS + cc * 8), vs + cc * 8, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  for (int i = 0; i < NBUF - WG && i < n_tiles; ++i) load_kv(t_begin + i, i);

  // stage Q (rotated) into shared memory: 8 dims of each rotary half per step, 16-byte loads
  constexpr int VH = HALF / 8;
  for (int idx = tid; idx < BM * VH; idx += NT) {
    const int r = idx / VH, d0 = (idx % VH) * 8;
    const int i = q0 + r;
    uint4 o1 = make_uint4(0, 0, 0, 0), o2 = o1;
    if (i < a.Lq) {
      const __nv_bfloat16* qr = Q + static_cast<long long>(i) * a.ldq;
      // L2 loads: in the persistent expert step, q was written by other CTAs in the same launch
      const uint4 u1 = __ldcg(reinterpret_cast<const uint4*>(qr + d0));
      const uint4 u2 = __ldcg(reinterpret_cast<const uint4*>(qr + d0 + HALF));
      const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u2);
      __nv_bfloat162* p1 = reinterpret_cast<__nv_bfloat162*>(&o1);
      __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&o2);
      if (a.cos) {
        const float4* c4 = reinterpret_cast<const float4*>(a.cos + static_cast<long long>(i) * HALF + d0);
        const float4* s4 = reinterpret_cast<const float4*>(a.sin + static_cast<long long>(i) * HALF + d0);
        const float4 ca = c4[0], cb = c4[1], sa = s4[0], sb = s4[1];
        const float cs[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
        const float sn[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x1 = __bfloat1622float2(h1[e]), x2 = __bfloat1622float2(h2[e]);
          const float c0 = cs[2 * e], c1 = cs[2 * e + 1], s0 = sn[2 * e], s1 = sn[2 * e + 1];
          p1[e] = __floats2bfloat162_rn(__fsub_rn(__fmul_rn(x1.x, c0), __fmul_rn(x2.x, s0)),
                                        __fsub_rn(__fmul_rn(x1.y, c1), __fmul_rn(x2.y, s1)));
          p2[e] = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(x2.x, c0), __fmul_rn(x1.x, s0)),
                                        __fadd_rn(__fmul_rn(x2.y, c1), __fmul_rn(x1.y, s1)));
        }
      } else {
        o1 = u1;
        o2 = u2;
      }
    }
    *reinterpret_cast<uint4*>(sQ + r * LDS + d0) = o1;
    *reinterpret_cast<uint4*>(sQ + r * LDS + d0 + HALF) = o2;
  }
  __syncthreads();

  uint32_t qf[HD / 16][4];
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const int row = warp * 16 + (lane & 15);
    const int col = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(smem_u32(sQ + row * LDS + col), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  float o[HD / 8][4];
#pragma unroll
  for (int t = 0; t < HD / 8; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int r0 = q0 + warp * 16 + (lane >> 2);  // this thread's two query rows
  const int r1 = r0 + 8;

  // rounds of WG tiles (one tile per round without warp groups)
  for (int first = 0; first < n_tiles; first += WG) {
    if (first + NBUF - 1 < n_tiles) {
      // refill the buffers of the previous round's tiles (every warp is past them: the round's
      // last barrier)
#pragma unroll
      for (int j = 0; j < WG; ++j) load_kv(t_begin + first + NBUF - WG + j, (first + NBUF - WG + j) % NBUF);
      cp_async_wait<NBUF - WG>();
    } else {
#pragma unroll
      for (int j = 0; j < WG; ++j)
        if (first + NBUF - WG + j < n_tiles) load_kv(t_begin + first + NBUF - WG + j, (first + NBUF - WG + j) % NBUF);
      cp_async_wait<0>();
    }
    __syncthreads();
    // the step's own keys in this round's tiles, rotated in place as the RoPE K/V cache kernel
    // would have written them (per-operation rounding, one rounding to bf16)
    bool rotated = false;
#pragma unroll
    for (int jt = 0; jt < WG; ++jt) {
      const long long j0 = static_cast<long long>(t_begin + first + jt) * BN;
      if (own && first + jt < n_tiles && j0 + BN > a.own_from) {
        rotated = true;
        const int r_lo = static_cast<int>(a.own_from > j0 ? a.own_from - j0 : 0);
        const int r_hi = static_cast<int>(a.Lk - j0 < BN ? a.Lk - j0 : BN);
        __nv_bfloat16* kt = sK + ((first + jt) % NBUF) * BN * LDS;
        for (int idx = tid; idx < (r_hi - r_lo) * HALF; idx += NT) {
          const int r = r_lo + idx / HALF, d = idx % HALF;
          const long long jr = j0 + r - a.own_from;
          const float k1 = __bfloat162float(kt[r * LDS + d]), k2 = __bfloat162float(kt[r * LDS + d + HALF]);
          const float c = a.k_cos[jr * HALF + d], sn = a.k_sin[jr * HALF + d];
          kt[r * LDS + d] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, sn)));
          kt[r * LDS + d + HALF] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(k2, c), __fmul_rn(k1, sn)));
        }
      }
    }
    if (rotated) __syncthreads();
    const int tile = first + grp;  // this group's tile of the round
    const int buf = tile % NBUF;
    if (WG == 1 || tile < n_tiles) {
    const __nv_bfloat16* k_s = sK + buf * BN * LDS;
    const __nv_bfloat16* v_s = sV + buf * BN * LDS;

    float s[BN / 8][4];
#pragma unroll
    for (int t = 0; t < BN / 8; ++t) s[t][0] = s[t][1] = s[t][2] = s[t][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int t2 = 0; t2 < BN / 16; ++t2) {
        const int key = t2 * 16 + (lane & 7) + (lane >> 4) * 8;
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(k_s + key * LDS + col), b0, b1, b2, b3);
        mma_bf16_16816(s[2 * t2], qf[kk], b0, b1);
        mma_bf16_16816(s[2 * t2 + 1], qf[kk], b2, b3);
      }
    }
    // scale, mask, row max. A tile whose keys all precede causal_from and Lk is visible to every
    // query (most of the prefix and expert tiles): no per-element mask there, same values.
    const int j0 = (t_begin + tile) * BN;
    float mx0 = -INFINITY, mx1 = -INFINITY;
    if (j0 + BN <= a.Lk && j0 + BN <= a.causal_from) {
#pragma unroll
      for (int t = 0; t < BN / 8; ++t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[t][e] *= a.scale_log2;
        mx0 = fmaxf(mx0, fmaxf(s[t][0], s[t][1]));
        mx1 = fmaxf(mx1, fmaxf(s[t][2], s[t][3]));
      }
    } else {
#pragma unroll
      for (int t = 0; t < BN / 8; ++t) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const long long j = j0 + t * 8 + (lane & 3) * 2 + (e & 1);
          const long long i = e < 2 ? r0 : r1;
          const bool vis = j < a.Lk && (j < a.causal_from || j <= i + a.q_offset);
          const float x = vis ? s[t][e] * a.scale_log2 : -INFINITY;
          s[t][e] = x;
          if (e < 2)
            mx0 = fmaxf(mx0, x);
          else
            mx1 = fmaxf(mx1, x);
        }
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = ex2(m0 - base0), al1 = ex2(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int t = 0; t < BN / 8; ++t) {
      const float p0 = ex2(s[t][0] - base0), p1 = ex2(s[t][1] - base0);
      const float p2 = ex2(s[t][2] - base1), p3 = ex2(s[t][3] - base1);
      ps0 += p0 + p1;
      ps1 += p2 + p3;
      pf[t / 2][(t & 1) * 2 + 0] = pack_bf16(p0, p1);
      pf[t / 2][(t & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int t = 0; t < HD / 8; ++t) {
      o[t][0] *= al0;
      o[t][1] *= al0;
      o[t][2] *= al1;
      o[t][3] *= al1;
    }
    // O += P V
#pragma unroll
    for (int j = 0; j < BN / 16; ++j) {
#pragma unroll
      for (int t2 = 0; t2 < HD / 16; ++t2) {
        const int key = j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = t2 * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(v_s + key * LDS + col), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * t2], pf[j], b0, b1);
        mma_bf16_16816(o[2 * t2 + 1], pf[j], b2, b3);
      }
    }
    }
    __syncthreads();  // these buffers are refilled at the top of the round after next
  }
  if constexpr (WG > 1) {
    // groups 1.. hand their running max, row sums (this thread's share) and output rows to group
    // 0 through the idle K/V ring; group 0 rescales and adds them in group order
    constexpr int XS = 4 + HD / 2;
    float* xch = reinterpret_cast<float*>(sK);
    if (grp > 0) {
      float* d = xch + ((grp - 1) * 128 + (tid & 127)) * XS;
      d[0] = m0, d[1] = m1, d[2] = l0, d[3] = l1;
#pragma unroll
      for (int t = 0; t < HD / 8; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[4 + t * 4 + e] = o[t][e];
    }
    __syncthreads();
    if (grp > 0) return;
#pragma unroll 1
    for (int g = 1; g < WG; ++g) {
      const float* d = xch + ((g - 1) * 128 + tid) * XS;
      const float n0 = fmaxf(m0, d[0]), n1 = fmaxf(m1, d[1]);
      const float b0 = n0 == -INFINITY ? 0.f : n0, b1 = n1 == -INFINITY ? 0.f : n1;
      const float sa0 = ex2(m0 - b0), sb0 = ex2(d[0] - b0), sa1 = ex2(m1 - b1), sb1 = ex2(d[1] - b1);
      l0 = l0 * sa0 + d[2] * sb0;
      l1 = l1 * sa1 + d[3] * sb1;
#pragma unroll
      for (int t = 0; t < HD / 8; ++t) {
        o[t][0] = o[t][0] * sa0 + d[4 + t * 4 + 0] * sb0;
        o[t][1] = o[t][1] * sa0 + d[4 + t * 4 + 1] * sb0;
        o[t][2] = o[t][2] * sa1 + d[4 + t * 4 + 2] * sb1;
        o[t][3] = o[t][3] * sa1 + d[4 + t * 4 + 3] * sb1;
      }
      m0 = n0;
      m1 = n1;
    }
  }

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const long long obase = bi * a.bo + static_cast<long long>(h) * HD;
  if constexpr (SPLIT) {
    // this split's unnormalised rows: O in the (now idle) K/V ring, (m, l) in the Q area
    constexpr int LDO = HD + 4;
    float* sO = reinterpret_cast<float*>(sK);
    float* sML = reinterpret_cast<float*>(sQ);   // [64][2]: running max, row sum
    const int lr0 = warp * 16 + (lane >> 2), lr1 = lr0 + 8;
    __syncthreads();  // every warp is done with the Q and K/V areas (a split may have had no tile)
#pragma unroll
    for (int t = 0; t < HD / 8; ++t) {
      const int col = t * 8 + (lane & 3) * 2;
      *reinterpret_cast<float2*>(sO + lr0 * LDO + col) = make_float2(o[t][0], o[t][1]);
      *reinterpret_cast<float2*>(sO + lr1 * LDO + col) = make_float2(o[t][2], o[t][3]);
    }
    if ((lane & 3) == 0) {
      sML[2 * lr0] = m0;
      sML[2 * lr0 + 1] = l0;
      sML[2 * lr1] = m1;
      sML[2 * lr1 + 1] = l1;
    }
    cluster_sync();
    // CTA `split` merges rows [split*64/S, (split+1)*64/S) over all splits, in split order. Per
    // item (row, 4 columns) every split's running max, row sum and O partial come in one round of
    // DSMEM loads (two items per thread and pass); each thread derives the merge weights of its
    // rows itself.
    const int rlo = split * BM / S, rhi = (split + 1) * BM / S, nr = rhi - rlo;
    const uint32_t o_addr = smem_u32(sO), ml_addr = smem_u32(sML);
    constexpr int IT = 2;
    for (int base = 0; base < nr * (HD / 4); base += IT * 128) {
      float ms[IT][8], ls[IT][8];
      float4 part[IT][8];
      int rr[IT], c4[IT];
      bool on[IT];
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        const int idx = base + it * 128 + tid;
        on[it] = idx < nr * (HD / 4);
        rr[it] = on[it] ? idx / (HD / 4) : 0;
        c4[it] = on[it] ? (idx % (HD / 4)) * 4 : 0;
        const int r = rlo + rr[it];
#pragma unroll
        for (int sp = 0; sp < 8; ++sp) {
          if (sp < S && on[it]) {
            const uint32_t pa = mapa_shared(ml_addr, static_cast<uint32_t>(sp)) + static_cast<uint32_t>(8 * r);
            ms[it][sp] = ld_cluster_f32(pa);
            ls[it][sp] = ld_cluster_f32(pa + 4);
            part[it][sp] = ld_cluster_f32x4(mapa_shared(o_addr, static_cast<uint32_t>(sp)) +
                                            static_cast<uint32_t>((r * LDO + c4[it]) * 4));
          }
        }
      }
#pragma unroll
      for (int it = 0; it < IT; ++it) {
        if (!on[it]) continue;
        float mx = -INFINITY;
#pragma unroll
        for (int sp = 0; sp < 8; ++sp)
          if (sp < S) mx = fmaxf(mx, ms[it][sp]);
        if (mx == -INFINITY) mx = 0.f;
        float l = 0.f;
#pragma unroll
        for (int sp = 0; sp < 8; ++sp) {
          if (sp < S) {
            ms[it][sp] = exp2f(ms[it][sp] - mx);
            l += ls[it][sp] * ms[it][sp];
          }
        }
        const float inv = 1.f / l;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < 8; ++sp) {
          if (sp < S) {
            const float wgt = ms[it][sp] * inv;
            acc.x += part[it][sp].x * wgt, acc.y += part[it][sp].y * wgt, acc.z += part[it][sp].z * wgt,
                acc.w += part[it][sp].w * wgt;
          }
        }
        const int row = q0 + rlo + rr[it];
        if (row < a.Lq) {
          const long long off = obase + static_cast<long long>(row) * a.ldo + c4[it];
          if (a.o_type == SO101_BF16) {
            __nv_bfloat162 hv[2] = {__floats2bfloat162_rn(acc.x, acc.y), __floats2bfloat162_rn(acc.z, acc.w)};
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.o) + off) = *reinterpret_cast<uint2*>(hv);
          } else {
            int8_t* pq = static_cast<int8_t*>(a.o) + off;
            pq[0] = quant_i8(acc.x, a.o_qscale);
            pq[1] = quant_i8(acc.y, a.o_qscale);
            pq[2] = quant_i8(acc.z, a.o_qscale);
            pq[3] = quant_i8(acc.w, a.o_qscale);
          }
        }
      }
    }
    cluster_sync_relaxed();  // peers keep their shared memory until every merge has read it
    return;
  }
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  if constexpr (TILE_OUT) {
    // this thread's columns t*8 + (lane&3)*2 + {0, 1} of a row are bytes (lane&3)*4 of chunk t
#pragma unroll
    for (int t = 0; t < HD / 8; ++t) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int row = half ? r1 : r0, lr = row - q0;
        const float inv = half ? inv1 : inv0;
        const uint32_t val = row < a.Lq ? pack_bf16(o[t][half * 2] * inv, o[t][half * 2 + 1] * inv) : 0u;
        *reinterpret_cast<uint32_t*>(o_tile + lr * 128 + ((t ^ (lr & 7)) << 4) + (lane & 3) * 4) = val;
      }
    }
  } else {
#pragma unroll
    for (int t = 0; t < HD / 8; ++t) {
      const int col = t * 8 + (lane & 3) * 2;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int row = half ? r1 : r0;
        if (row >= a.Lq) continue;
        const float x0 = o[t][half * 2] * (half ? inv1 : inv0);
        const float x1 = o[t][half * 2 + 1] * (half ? inv1 : inv0);
        const long long off = obase + static_cast<long long>(row) * a.ldo + col;
        if (a.o_type == SO101_BF16) {
          *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(a.o) + off) = __floats2bfloat162_rn(x0, x1);
        } else {
          int8_t* p = static_cast<int8_t*>(a.o) + off;
          p[0] = quant_i8(x0, a.o_qscale);
          p[1] = quant_i8(x1, a.o_qscale);
        }
      }
    }
  }
}

// Four CTAs per SM where the registers allow it (head_dim <= 64: the unsplit kernel of the batched
// prefix and expert fits 128 registers).
template <int HD, bool SPLIT>
__global__ void __launch_bounds__(128, HD <= 64 ? 4 : 1) attention_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  grid_dep_launch();
  grid_dep_wait();
  const int S = SPLIT ? a.kv_splits : 1;
  const int split = S > 1 ? static_cast<int>(blockIdx.x % S) : 0;
  const int q0 = (S > 1 ? blockIdx.x / S : blockIdx.x) * 64;
  attention_body<HD, SPLIT>(a, split, q0, blockIdx.y, blockIdx.z, smem_raw);
}

}  // namespace so101
