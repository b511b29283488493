// Attention fused with its output projection and residual, for the few query rows of the action
// expert at batch 1: y = residual + attention(q, k, v) @ W_o^T, one launch instead of an attention
// launch followed by a GEMM launch.
//
// The output projection's K dimension is the heads: y = sum over heads h of O_h W_o[:, h]^T, with
// O_h the (rows x 64) attention output of head h and W_o[:, h] the 64 columns of W_o that read it.
// So the grid is clusters of nq CTAs (one per query head, cluster rank = head) per 128-feature
// output tile and 64-row query block. Each CTA
//   1  issues the TMA load of its W_o block (128 features x 64, SWIZZLE_128B) before waiting for
//      the previous grid: the weights do not depend on it;
//   2  runs the attention of its head over all keys, writing the normalised rows as bf16 straight
//      into the MMA's B operand tile in shared memory (the same bf16 rounding the unfused path
//      applies before storing them): the mma.sync flash loop of attention_tile.cuh (a six-tile
//      K/V ring; two or three warp groups taking the tiles in turn, merged at the end), or, by
//      default when the keys fit six 64-key tiles (SO101_ATTN_O_TC=0 turns it off), on tcgen05
//      (attention_head_tc);
//   3  issues one M=128, N=64, K=64 tcgen05.mma: its head's fp32 partial (features x tokens) in
//      TMEM, staged to shared memory;
//   4  after a cluster barrier, sums whole tokens over the nq partials through DSMEM in head
//      order and runs the residual epilogue (token_reduce.cuh): fp32 row, bf16 copy scaled by the
//      next RMSNorm's weight, the token's sum of squares over the tile (statistics slot = tile).
// Redundancy: every output tile's cluster recomputes the attention (a few microseconds of tensor
// work on the key/value rows that L2 holds); what it saves is a dependent launch and the round
// trip of the attention output through global memory.
#include <cstdlib>
#include <mutex>

#include "attention_tile.cuh"
#include "tc_attn.cuh"
#include "token_reduce.cuh"

namespace so101 {

struct AttnOArgs {
  AttnArgs at;       // at.o unused
  TokenEpilogue ep;  // output tile epilogue
  int q_blocks;      // 64-row query blocks per problem
  int tc;            // 1: the attention on tcgen05 (every query block's keys fit kAoTcTiles tiles)
  int* status;
};

constexpr int kAoBuf = 6;                               // K/V ring: the expert's 5 key tiles at once
constexpr int kAoMaxHeads = 16;                         // largest (non-portable) cluster
constexpr int kAoOffW = 0;                              // W_o block: 128 x 64 bf16, 16 KB
constexpr int kAoOffO = 128 * 128;                      // O tile: 64 x 64 bf16, 8 KB
constexpr int kAoOffAttn = kAoOffO + 64 * 128;          // attention_body's area, then the partial
constexpr int kAoOffBar = kAoOffAttn + attention_smem_bytes<64, kAoBuf>();
constexpr int kAoSmem = kAoOffBar + 64 + 1024;          // + 1024-byte alignment of the base
static_assert(attention_smem_bytes<64, kAoBuf>() >= 64 * 128 * 4, "the fp32 partial reuses the attention area");

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ attention of one head on tcgen05
// Query rows [q0, q0 + 64) of head h against all keys it can see, in one pass (no online rescaling):
//   1  every thread: K and V rows into shared memory (cp.async, K-major SWIZZLE_128B rows of 128
//      bytes, 64-key tiles back to back; rows past Lk zero), the step's own keys loaded, rotated
//      (the RoPE K/V cache kernel's arithmetic) and stored by the threads; warp group 0: the query
//      rows, rotated, into the Q operand tile (rows 64..127 zero);
//   2  one thread: S = Q K^T, one M = 128, N = 64, K = 64 MMA per key tile, into TMEM columns
//      [64 t, 64 t + 64);
//   3  the warps of TMEM lanes 0..63 (G per lane quarter, key tiles dealt round robin): the row
//      maximum of the scaled, masked scores, exchanged through shared memory; then
//      p = 2^(s * scale - max) rounded to bf16 and the row sums; once every score is read, P is
//      written over S (two keys per column, columns [32 t, 32 t + 32));
//   4  one thread: O = P V (A = P from TMEM, B = V MN-major, K = 16 per MMA) into columns
//      [kAoTcColO, +64);
//   5  the first warp of each lane quarter: O / l (l summed over the G partial sums in order) as bf16
//      into the output tile (the mma.sync path's layout: row r, chunk c at c ^ (r % 8); rows at or
//      past Lq zero).
// TMEM: 512 columns (S or P up to 384, O at 384). Shared memory: the attention area of the kernel.
constexpr int kAoTcTiles = 6;  // 384 keys
constexpr uint32_t kAoTcColO = 384;
constexpr int kAoTcOffQ = 0;
constexpr int kAoTcOffK = kAoTcOffQ + 128 * 128;
constexpr int kAoTcOffV = kAoTcOffK + kAoTcTiles * 64 * 128;
constexpr int kAoTcOffX = kAoTcOffV + kAoTcTiles * 64 * 128;  // [2][3][64] fp32: row maxima, row sums
static_assert(kAoTcOffX + 2 * 3 * 64 * 4 <= attention_smem_bytes<64, kAoBuf>(), "the tcgen05 attention fits the area");

// key tiles of 64 keys that query rows [q0, q0 + 64) can see (attention_body's count)
__device__ __forceinline__ int ao_key_tiles(const AttnArgs& a, int q0) {
  long long last = a.causal_from - 1;
  const long long diag = static_cast<long long>(q0 + 63) + a.q_offset;
  if (diag > last) last = diag;
  if (last > a.Lk - 1) last = a.Lk - 1;
  return static_cast<int>((last + 64) / 64);
}

// bf16 row pieces: chunks c (dims 8c..8c+7) and c + 4 (their rotary partners) rotated by the eight
// cos/sin values of those dims, per-operation rounding, one rounding to bf16.
__device__ __forceinline__ void ao_rotate(const uint4& u1, const uint4& u2, const float* cs, const float* sn, uint4& o1,
                                          uint4& o2) {
  const float4 ca = __ldg(reinterpret_cast<const float4*>(cs)), cb = __ldg(reinterpret_cast<const float4*>(cs + 4));
  const float4 sa = __ldg(reinterpret_cast<const float4*>(sn)), sb = __ldg(reinterpret_cast<const float4*>(sn + 4));
  const float cv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
  const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
  const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u2);
  __nv_bfloat162* p1 = reinterpret_cast<__nv_bfloat162*>(&o1);
  __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&o2);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x1 = __bfloat1622float2(h1[e]), x2 = __bfloat1622float2(h2[e]);
    const float c0 = cv[2 * e], c1 = cv[2 * e + 1], s0 = sv[2 * e], s1 = sv[2 * e + 1];
    p1[e] = __floats2bfloat162_rn(__fsub_rn(__fmul_rn(x1.x, c0), __fmul_rn(x2.x, s0)),
                                  __fsub_rn(__fmul_rn(x1.y, c1), __fmul_rn(x2.y, s1)));
    p2[e] = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(x2.x, c0), __fmul_rn(x1.x, s0)),
                                  __fadd_rn(__fmul_rn(x2.y, c1), __fmul_rn(x1.y, s1)));
  }
}

// All 128 G threads call it. False when an MMA wait ran out (SO101_ERR_TIMEOUT recorded); the
// output tile is then not written.
template <int G>
__device__ __forceinline__ bool attention_head_tc(const AttnArgs& a, int q0, int h, int bi, uint8_t* area,
                                                  uint8_t* o_tile, uint32_t tmem, uint64_t* s_done, uint64_t* o_done,
                                                  int* status) {
  constexpr int NT = 128 * G;
  constexpr int TPW = (kAoTcTiles + G - 1) / G;  // key tiles per softmax warp
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int kvh = h / (a.nq / a.nkv);
  const __nv_bfloat16* K = a.k + bi * a.bk + static_cast<long long>(kvh) * 64;
  const __nv_bfloat16* V = a.v + bi * a.bv + static_cast<long long>(kvh) * 64;
  const bool own = a.k_own != nullptr;
  const __nv_bfloat16* K_own = own ? a.k_own + bi * a.b_own + static_cast<long long>(kvh) * 64 : nullptr;
  const __nv_bfloat16* V_own = own ? a.v_own + bi * a.b_own + static_cast<long long>(kvh) * 64 : nullptr;
  const int n_tiles = ao_key_tiles(a, q0);
  const int n_rows = n_tiles * 64;
  const long long own_from = own ? a.own_from : a.Lk;
  uint8_t* q_s = area + kAoTcOffQ;
  uint8_t* k_s = area + kAoTcOffK;
  uint8_t* v_s = area + kAoTcOffV;
  float* x_max = reinterpret_cast<float*>(area + kAoTcOffX);  // [G][64]
  float* x_sum = x_max + 3 * 64;                               // [G][64]

  // 1. keys and values (own keys are rotated below), queries
  for (int c = t; c < n_rows * 8; c += NT) {
    const int j = c >> 3, cc = c & 7;
    const bool ok = j < a.Lk;
    const long long jj = ok ? j : 0;
    const bool mine = jj >= own_from;
    const uint32_t off = static_cast<uint32_t>(j * 128 + ((cc ^ (j & 7)) << 4));
    if (!mine || !ok) cp_async16(smem_u32(k_s) + off, K + jj * a.ldk + cc * 8, ok ? 16 : 0);
    const __nv_bfloat16* vs = mine ? V_own + (jj - own_from) * a.ld_own : V + jj * a.ldv;
    cp_async16(smem_u32(v_s) + off, vs + cc * 8, ok ? 16 : 0);
  }
  cp_async_commit();
  if (t < 128) {
    const int i = q0 + t;
    uint4 out[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) out[c] = make_uint4(0u, 0u, 0u, 0u);
    if (t < 64 && i < a.Lq) {
      const uint4* qr = reinterpret_cast<const uint4*>(a.q + bi * a.bq + static_cast<long long>(i) * a.ldq + h * 64);
      uint4 u[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) u[c] = __ldcg(qr + c);
      if (a.cos) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          ao_rotate(u[c], u[c + 4], a.cos + static_cast<long long>(i) * 32 + 8 * c,
                    a.sin + static_cast<long long>(i) * 32 + 8 * c, out[c], out[c + 4]);
      } else {
#pragma unroll
        for (int c = 0; c < 8; ++c) out[c] = u[c];
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(q_s + t * 128 + ((c ^ (t & 7)) << 4)) = out[c];
  }
  if (own) {
    const int j_lo = static_cast<int>(own_from), j_hi = min(a.Lk, n_rows);
    for (int idx = t; idx < (j_hi - j_lo) * 4; idx += NT) {
      const int j = j_lo + (idx >> 2), c = idx & 3;
      const long long jr = j - own_from;
      const uint4* kr = reinterpret_cast<const uint4*>(K_own + jr * a.ld_own);
      uint4 o1, o2;
      ao_rotate(__ldcg(kr + c), __ldcg(kr + c + 4), a.k_cos + jr * 32 + 8 * c, a.k_sin + jr * 32 + 8 * c, o1, o2);
      *reinterpret_cast<uint4*>(k_s + j * 128 + ((c ^ (j & 7)) << 4)) = o1;
      *reinterpret_cast<uint4*>(k_s + j * 128 + (((c + 4) ^ (j & 7)) << 4)) = o2;
    }
  }
  cp_async_wait<0>();
  fence_async_smem();  // cp.async and plain stores, before the tensor core reads them
  tc_fence_before();
  __syncthreads();

  // 2. S = Q K^T, issued by warp 0's elected lane (warp-uniform descriptors)
  if ((t >> 5) == 0) {
    tc_fence_after();
    constexpr uint32_t ID_S = idesc_attn(64, 0);
    const uint64_t qd = sw128_desc(smem_u32(q_s));
    if (elect_one()) {
      for (int tile = 0; tile < n_tiles; ++tile) {
        const uint64_t kd = sw128_desc(smem_u32(k_s + tile * 64 * 128));
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16(tmem + 64 * tile, qd + 2 * k, kd + 2 * k, ID_S, k > 0 ? 1u : 0u);
      }
      mma_commit(s_done);
    }
    __syncwarp();
  }

  // 3. softmax over TMEM lanes 0..63: quarter q = warp % 4 < 2, warp group g = warp / 4
  const int quarter = warp & 3, g = warp >> 2;
  const int row = quarter * 32 + lane, i = q0 + row;
  const bool soft = quarter < 2;
  const bool live = soft && i < a.Lq;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
  const float sc = a.scale_log2;
  // keys [0, vis_end) are visible to row i
  long long vis_end = static_cast<long long>(i) + a.q_offset + 1;
  if (vis_end < a.causal_from) vis_end = a.causal_from;
  if (vis_end > a.Lk) vis_end = a.Lk;
  bool ok = true;
  if (soft) {
    ok = __all_sync(0xffffffffu, mbar_wait(s_done, 0, status) ? 1 : 0) != 0;
    tc_fence_after();
    float m = -INFINITY;
    if (ok) {
      for (int u = 0; u < TPW; ++u) {
        const int tile = g + u * G;
        if (tile >= n_tiles) break;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t sv[32];
          tmem_ld32(lane_base + 64 * tile + 32 * half, sv);
          tmem_ld_wait();
          const int j0 = 64 * tile + 32 * half;
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (j0 + e < vis_end) m = fmaxf(m, __uint_as_float(sv[e]) * sc);
        }
      }
    }
    x_max[g * 64 + row] = m;
  }
  __syncthreads();
  uint32_t pk[TPW][32];
  if (soft) {
    float mx = x_max[row];
#pragma unroll
    for (int gg = 1; gg < G; ++gg) mx = fmaxf(mx, x_max[gg * 64 + row]);
    const float neg_m = (live && mx != -INFINITY) ? -mx : 0.f;
    float ls = 0.f;
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tile = g + u * G;
      if (tile >= n_tiles || !ok) break;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t sv[32];
        tmem_ld32(lane_base + 64 * tile + 32 * half, sv);
        tmem_ld_wait();
        const int j0 = 64 * tile + 32 * half;
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x0, x1;
          fma2(x0, x1, __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), sc, neg_m);
          const float p0 = (live && j0 + e < vis_end) ? ex2(x0) : 0.f;
          const float p1 = (live && j0 + e + 1 < vis_end) ? ex2(x1) : 0.f;
          ls += p0 + p1;
          pk[u][16 * half + (e >> 1)] = bf16x2(p0, p1);
        }
      }
    }
    x_sum[g * 64 + row] = ls;
  }
  tc_fence_before();
  __syncthreads();  // every score is read: P may overwrite S
  if (soft && ok) {
    tc_fence_after();
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tile = g + u * G;
      if (tile >= n_tiles) break;
      tmem_st16(lane_base + 32 * tile, pk[u]);
      tmem_st16(lane_base + 32 * tile + 16, pk[u] + 16);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();

  // 4. O = P V, issued by warp 0's elected lane (ok is warp-uniform there)
  if ((t >> 5) == 0 && ok) {
    tc_fence_after();
    constexpr uint32_t ID_O = idesc_attn(64, 1);
    const uint64_t vd = sw128_desc(smem_u32(v_s));
    if (elect_one()) {
      for (int k = 0; k < 4 * n_tiles; ++k)
        mma_f16_ta(tmem + kAoTcColO, tmem + 8 * k, vd + static_cast<uint64_t>(k) * (2048 >> 4), ID_O, k > 0 ? 1u : 0u);
      mma_commit(o_done);
    }
    __syncwarp();
  }

  // 5. O / l into the output tile
  if (soft && g == 0) {
    ok = ok && __all_sync(0xffffffffu, mbar_wait(o_done, 0, status) ? 1 : 0) != 0;
    tc_fence_after();
    if (ok) {
      uint32_t ov[64];
      tmem_ld32(lane_base + kAoTcColO, ov);
      tmem_ld32(lane_base + kAoTcColO + 32, ov + 32);
      tmem_ld_wait();
      float l = x_sum[row];
#pragma unroll
      for (int gg = 1; gg < G; ++gg) l += x_sum[gg * 64 + row];
      const float inv = live ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float* v = reinterpret_cast<const float*>(ov) + 8 * c;
        const uint4 val = live ? make_uint4(bf16x2(v[0] * inv, v[1] * inv), bf16x2(v[2] * inv, v[3] * inv),
                                            bf16x2(v[4] * inv, v[5] * inv), bf16x2(v[6] * inv, v[7] * inv))
                               : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(o_tile + row * 128 + ((c ^ (row & 7)) << 4)) = val;
      }
    }
  }
  return ok;
}

// G warp groups of 128 threads take the key tiles in turn (attention_body's WG).
template <int G>
__global__ void __launch_bounds__(128 * G, 1) attention_o_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                 const AttnOArgs a) {
  constexpr int kAoThreads = 128 * G;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + kAoOffBar);
  uint64_t* mma_done = w_full + 1;
  uint64_t* s_done = mma_done + 1;  // tcgen05 attention: the scores, then the output rows
  uint64_t* o_done = s_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);
  const int t = threadIdx.x, warp = t >> 5;
  const int h = blockIdx.x, tile = blockIdx.y;
  const int qb = blockIdx.z % a.q_blocks, bi = blockIdx.z / a.q_blocks;
  const int q0 = qb * 64;
  const uint32_t kCols = a.tc ? 512 : 64;

  if (t == 0) {
    mbar_init(w_full, 1);
    mbar_init(mma_done, 1);
    mbar_init(s_done, 1);
    mbar_init(o_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (t == 0) {
    tma_prefetch_desc(&tm_w);
    mbar_arrive_expect_tx(w_full, 128 * 128);
    tma_load_2d(smem + kAoOffW, &tm_w, w_full, h * 64, tile * 128, policy_evict_normal());
  }
  grid_dep_launch();
  grid_dep_wait();
  const int nv = min(64, a.at.Lq - q0);  // valid tokens of this query block
  const long long row0 = static_cast<long long>(bi) * a.at.Lq + q0;
  const TokenPrefetch pf = token_prefetch<kAoThreads>(a.ep, a.at.nq, nv, row0, tile);

  if (a.tc)
    attention_head_tc<G>(a.at, q0, h, bi, smem + kAoOffAttn, smem + kAoOffO, tmem, s_done, o_done, a.status);
  else
    attention_body<64, false, true, kAoBuf, G>(a.at, 0, q0, h, bi, smem + kAoOffAttn, smem + kAoOffO);
  fence_async_smem();  // the O tile's generic-proxy stores, before the tensor core reads them
  __syncthreads();
  if (warp == 0) {
    // warp 0 waits together, its elected lane issues (warp-uniform descriptors)
    if (__all_sync(0xffffffffu, mbar_wait(w_full, 0, a.status))) {
      tc_fence_after();
      const uint64_t ad = sw128_desc(smem_u32(smem + kAoOffW)), bd = sw128_desc(smem_u32(smem + kAoOffO));
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k) mma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc_bf16(128, 64), k > 0 ? 1u : 0u);
        mma_commit(mma_done);
      }
    } else if (elect_one()) {
      mbar_arrive(mma_done);  // the weights never came: unwind through the cluster barriers
    }
  }
  __syncwarp();
  const bool mma_ok = __all_sync(0xffffffffu, mbar_wait(mma_done, 0, a.status) ? 1 : 0) != 0;
  tc_fence_after();

  // this head's partial, column-major (a token's 128 features contiguous), over the attention area
  float* part = reinterpret_cast<float*>(smem + kAoOffAttn);
  if (mma_ok) {
    // thread t: TMEM lane t % 128 (warp w reads lanes 32 (w % 4) ..), 16-token chunks c with
    // c / 16 = t / 128 modulo the group count
    const int tl = t & 127;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll 1
    for (int c = (t >> 7) * 16; c < nv; c += 16 * G) {
      uint32_t r[16];
      tmem_ld16(lane_addr + c, r);
      tmem_ld_wait(r);
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(c + j) * 128 + tl] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  cluster_sync();

  cluster_token_reduce<kAoMaxHeads, kAoThreads>(a.ep, part, a.at.nq, nv, row0, tile, pf);
  cluster_sync_relaxed();  // no CTA leaves while a peer still reads its partial
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

}  // namespace so101

using namespace so101;

namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// The attention of so101_attention_o runs on tcgen05 when the keys fit six 64-key tiles, unless
// SO101_ATTN_O_TC=0 (read per call: the engine calls it while it records its programs) selects the
// mma.sync flash loop. With its MMAs issued by an elected lane of a warp-uniform warp 0 the tcgen05
// form measured denoise 5.155 against 5.286 ms per batch-1 chunk; issued by one thread it had been
// 0.1 ms per chunk slower than the mma.sync loop.
bool ao_tc_enabled() {
  const char* e = std::getenv("SO101_ATTN_O_TC");
  return !(e && e[0] == '0');
}

// Whether a cluster of `heads` CTAs of attention_o_kernel<G> can be resident at all (non-portable
// sizes above 8 depend on the GPU); cached per group count and cluster size.
template <int G>
int cluster_fits(int heads, cudaStream_t stream) {
  static int known[kAoMaxHeads + 1] = {};  // 0 unknown, 1 fits, -1 does not
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_o_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAoSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_o_kernel<G>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  if (known[heads] == 0) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(heads, 1, 1);
    lc.blockDim = dim3(128 * G);
    lc.dynamicSmemBytes = kAoSmem;
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = heads;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int clusters = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, attention_o_kernel<G>, &lc);
    if (e != cudaSuccess) return launch_error(e);
    known[heads] = clusters > 0 ? 1 : -1;
  }
  return known[heads] > 0 ? SO101_OK : SO101_ERR_ARG;
}

}  // namespace

extern "C" int so101_attention_o(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                 int64_t Lq, int64_t Lk, int nq, int nkv, int hd, int64_t causal_from,
                                 int64_t q_offset, const float* cos, const float* sin, int batch, int64_t bq,
                                 int64_t bk, int64_t bv, const void* k_own, const void* v_own, int64_t ld_own,
                                 int64_t b_own, int64_t own_from, const float* k_cos, const float* k_sin,
                                 const void* w_o, int64_t ldw, int64_t n_out, float* y, int64_t ldy,
                                 const float* residual, int64_t ldr, void* y16, int64_t ld16, const float* y16_scale,
                                 float* stat_ss, int64_t stat_ld, cudaStream_t stream) {
  if (!q || !k || !v || !w_o || !y || Lq <= 0 || Lk <= 0 || nkv <= 0 || nq <= 0 || nq % nkv || batch <= 0)
    return SO101_ERR_ARG;
  if (hd != 64 || nq > kAoMaxHeads || n_out <= 0 || n_out % 4 || n_out > (1 << 20)) return SO101_ERR_ARG;
  if (Lq > (1 << 24) || Lk > (1 << 30)) return SO101_ERR_ARG;
  if ((cos == nullptr) != (sin == nullptr)) return SO101_ERR_ARG;
  const long long q_blocks = (Lq + 63) / 64;
  if (q_blocks * batch > 65535 || (n_out + 127) / 128 > 65535) return SO101_ERR_ARG;
  // attention operands, as so101_attention checks them
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (ldq * 2) % 16 || (ldk * 2) % 16 || (ldv * 2) % 16 ||
      (bq * 2) % 16 || (bk * 2) % 16 || (bv * 2) % 16)
    return SO101_ERR_ARG;
  if (cos && (!aligned16(cos) || !aligned16(sin))) return SO101_ERR_ARG;
  if (k_own) {
    if (!v_own || !k_cos || !k_sin || own_from < 0 || own_from > Lk || !aligned16(k_own) || !aligned16(v_own) ||
        (ld_own * 2) % 16 || (b_own * 2) % 16)
      return SO101_ERR_ARG;
  }
  // projection and epilogue: 16-byte weight rows for TMA, float4 / 4 x bf16 row pieces
  if (!aligned16(w_o) || (ldw * 2) % 16 || ldw < static_cast<int64_t>(nq) * hd) return SO101_ERR_ARG;
  if (!aligned16(y) || ldy % 4 || ldy < n_out) return SO101_ERR_ARG;
  if (residual && (!aligned16(residual) || ldr % 4 || ldr < n_out)) return SO101_ERR_ARG;
  if (y16 && (reinterpret_cast<uintptr_t>(y16) % 8 || ld16 % 4 || ld16 < n_out)) return SO101_ERR_ARG;
  if (y16_scale && !aligned16(y16_scale)) return SO101_ERR_ARG;
  const int tiles = static_cast<int>((n_out + 127) / 128);
  if (stat_ss && stat_ld < tiles) return SO101_ERR_ARG;

  EncodeFn enc = encode_fn();
  if (!enc) return SO101_ERR_DRIVER;
  CUtensorMap tm;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(nq) * hd, static_cast<cuuint64_t>(n_out)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw) * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w_o), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SO101_ERR_ARG;
  }
  // key tiles of the last query block (attention_body's count): three warp groups when that takes
  // fewer rounds than two (the expert's 291 self-attention keys: 5 tiles, 2 rounds against 3)
  long long last = causal_from - 1;
  if ((q_blocks - 1) * 64 + 63 + q_offset > last) last = (q_blocks - 1) * 64 + 63 + q_offset;
  if (last > Lk - 1) last = Lk - 1;
  const long long key_tiles = (last + 64) / 64;
  const int groups = (key_tiles + 2) / 3 < (key_tiles + 1) / 2 ? 3 : 2;
  const int fit = groups == 3 ? cluster_fits<3>(nq, stream) : cluster_fits<2>(nq, stream);
  if (fit != SO101_OK) return fit;

  AttnOArgs a;
  AttnArgs& at = a.at;
  at.q = static_cast<const __nv_bfloat16*>(q);
  at.k = static_cast<const __nv_bfloat16*>(k);
  at.v = static_cast<const __nv_bfloat16*>(v);
  at.o = nullptr;
  at.ldq = ldq;
  at.ldk = ldk;
  at.ldv = ldv;
  at.ldo = 0;
  at.bq = bq;
  at.bk = bk;
  at.bv = bv;
  at.bo = 0;
  at.o_type = SO101_BF16;
  at.o_qscale = 0.f;
  at.Lq = static_cast<int>(Lq);
  at.Lk = static_cast<int>(Lk);
  at.nq = nq;
  at.nkv = nkv;
  at.causal_from = causal_from;
  at.q_offset = q_offset;
  at.cos = cos;
  at.sin = sin;
  at.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(hd)));
  at.kv_splits = 1;
  at.k_own = static_cast<const __nv_bfloat16*>(k_own);
  at.v_own = static_cast<const __nv_bfloat16*>(v_own);
  at.ld_own = ld_own;
  at.b_own = b_own;
  at.own_from = own_from;
  at.k_cos = k_cos;
  at.k_sin = k_sin;
  a.ep = TokenEpilogue{y, ldy, residual, ldr, static_cast<__nv_bfloat16*>(y16), ld16, y16_scale, stat_ss, stat_ld,
                       static_cast<int>(n_out)};
  a.q_blocks = static_cast<int>(q_blocks);
  // (the tcgen05 path reads the own keys' rotary tables as float4 rows)
  const bool tables16 = !k_own || (aligned16(k_cos) && aligned16(k_sin));
  a.tc = (key_tiles <= kAoTcTiles && tables16 && ao_tc_enabled()) ? 1 : 0;
  a.status = status_ptr();

  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(nq, tiles, static_cast<unsigned>(q_blocks * batch));
  lc.blockDim = dim3(128 * groups);
  lc.dynamicSmemBytes = kAoSmem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nq;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = groups == 3 ? cudaLaunchKernelEx(&lc, attention_o_kernel<3>, tm, a)
                                    : cudaLaunchKernelEx(&lc, attention_o_kernel<2>, tm, a);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}
