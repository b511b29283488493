// Masked grouped-query attention on tcgen05 for the prefix pass and the action expert with many
// observations (the batched engine): head_dim 64, RoPE on the queries, the block-causal mask
// `key j visible to query i  <=>  j < Lk and (j < causal_from or j <= i + q_offset)`.
//
// The kernel is written for NG groups of 128 query rows per CTA (MMA M = 128); the plan runs one:
// either one query head's positions [128 b, 128 b + 128) (the prefix: 241 rows per head in two
// blocks), or the query heads of one kv head stacked (the expert: two of its three 50-row heads),
// so that each key tile serves every query head that reads it. Per 128-key tile j:
//   warp 0 (one thread)  TMA: K_j and V_j of this observation's kv head into two-stage rings
//   warp 1 (one thread)  S_g = Q_g K_j^T (M 128, N 128, K 64) -> TMEM; O_g += P_g V_j with P_g
//                        read from TMEM (the SigLIP kernel's scheme, attention_tc.cu)
//   warps 2-5            first the queries: each thread loads its row, rotates it in fp32 (the
//                        reference's rope, rounded once to bf16) and writes it into the swizzled
//                        Q operand tile; then the softmax of its row, one TMEM lane, with the mask
//                        computed from the key index, and at the end O / l to the output rows.
// Key rows past Lk inside the last tile belong to the next observation (or are zero-filled past
// the tensor's end): the mask gives them probability zero. The row maximum follows the SigLIP
// kernel's stale-maximum rule (raised only when a tile exceeds it by more than 2^8).
#include "tc_attn.cuh"

namespace so101 {

struct GqaArgs {
  const __nv_bfloat16* q;  // query rows, head h at columns [64 h, 64 h + 64)
  long long ldq, bq;       // row stride and per-observation stride (elements)
  __nv_bfloat16* o;
  long long ldo, bo;
  int Lq, Lk, nq, nkv;
  int heads_per_cta;       // query heads stacked in one CTA (q_blocks == 1 when > 1)
  int q_blocks;            // 256-row blocks per query head
  long long k_rows, v_rows;  // rows per observation in the K and V maps
  long long causal_from, q_offset;
  const float* cos;        // (Lq, 32) rotary tables of the queries (null: no rotation)
  const float* sin;
  float scale_log2;
  int* status;
  // Keys j >= own_from (at most kGqOwn of them) are the step's own rows, read from k_own / v_own
  // (row stride ld_own, observation stride b_own, kv head at columns 64 kvh) instead of the K / V
  // maps, the keys rotated by k_cos / k_sin (row j - own_from) as the RoPE K/V cache kernel would;
  // the cache rows there are never read. k_own == nullptr: own_from = Lk, none.
  const __nv_bfloat16* k_own = nullptr;
  const __nv_bfloat16* v_own = nullptr;
  long long ld_own = 0, b_own = 0, own_from = 0;
  const float* k_cos = nullptr;
  const float* k_sin = nullptr;
};

constexpr int kGqRows = 128;
constexpr int kGqKeys = 128;
constexpr int kGqHd = 64;
constexpr int kGqTile = kGqRows * kGqHd * 2;  // 16 KB
constexpr int kGqOwn = 64;                     // most own keys: one 64-key tile (the expert's 50)
constexpr float kGqStaleMax = 8.f;
constexpr int kGqBarBytes = 512;

// NG query groups of 128 rows per CTA. One: 256 TMEM columns and a two-stage ring, two CTAs per
// SM, so the short, latency-bound CTAs overlap. (Two groups per CTA, all 512 columns, a four-stage
// ring and one CTA per SM, measured 86.7 against 70.6 us for the prefix's attention at 64
// observations, so the plan no longer picks them.)
template <int NG>
struct GqCfg {
  static constexpr int kStages = NG == 2 ? 4 : 2;
  static constexpr int kThreads = 32 * (2 + 4 * NG);
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + NG * kGqTile;
  static constexpr int kOffV = kOffK + kStages * kGqTile;
  static constexpr int kOffOwnK = kOffV + kStages * kGqTile;  // the own keys, rotated (64 rows)
  static constexpr int kOffOwnV = kOffOwnK + kGqOwn * 128;    // the own values
  static constexpr int kOffBar = kOffOwnV + kGqOwn * 128;
  static constexpr int kSmem = kOffBar + kGqBarBytes + 1024;
  static constexpr uint32_t kCols = NG == 2 ? 512 : 256;
  // TMEM columns: S (128 per group), P (64 per group: 128 bf16 keys in pairs), O (64 per group)
  static constexpr uint32_t kColS = 0, kColP = NG * 128, kColO = NG * 128 + NG * 64;
};
static_assert((1 + 4 * 4 + 8) * 8 + 4 <= kGqBarBytes, "barrier region");
static_assert(2 * GqCfg<1>::kSmem <= 232448, "shared memory per CTA / SM");

// Two 8-dim chunks of a bf16 row, u1 (dims 8c..8c+7) and u2 (their rotary partners 32 later),
// rotated by cos / sin (8 floats each, 16-byte aligned): per-operation rounding, one rounding to
// bf16, as the reference's rope and the RoPE K/V cache kernel.
__device__ __forceinline__ void gq_rotate(const uint4& u1, const uint4& u2, const float* cs, const float* sn, uint4& o1,
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

// Query row r of this CTA: its head and position, or false for a padding row. One head per CTA:
// positions [rows qb, rows (qb + 1)); several: heads head0 .. head0 + n_heads - 1 stacked, Lq rows
// each.
template <int NG>
__device__ __forceinline__ bool gqa_row(const GqaArgs& a, int r, int head0, int n_heads, int qb, int& head,
                                        int& pos) {
  if (a.heads_per_cta == 1) {
    head = head0;
    pos = qb * NG * kGqRows + r;
  } else {
    head = head0 + r / a.Lq;
    pos = r % a.Lq;
    if (r >= n_heads * a.Lq) return false;
  }
  return pos < a.Lq;
}

template <int NG>
__global__ void __launch_bounds__(GqCfg<NG>::kThreads, NG == 1 ? 2 : 1)
    attention_gqa_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const GqaArgs a) {
  using Cfg = GqCfg<NG>;
  constexpr int kGqStages = Cfg::kStages;
  constexpr int kGqOffQ = Cfg::kOffQ, kGqOffK = Cfg::kOffK, kGqOffV = Cfg::kOffV;
  constexpr uint32_t kGqColS = Cfg::kColS, kGqColP = Cfg::kColP, kGqColO = Cfg::kColO;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
  uint64_t* q_full = bar;                      // [1] the softmax warps wrote their Q rows
  uint64_t* k_full = bar + 1;                  // [kGqStages]
  uint64_t* k_empty = k_full + kGqStages;      // [kGqStages]
  uint64_t* v_full = k_empty + kGqStages;      // [kGqStages]
  uint64_t* v_empty = v_full + kGqStages;      // [kGqStages]
  uint64_t* s_full = v_empty + kGqStages;      // [2]
  uint64_t* s_free = s_full + 2;               // [2]
  uint64_t* p_full = s_free + 2;               // [2]
  uint64_t* o_full = p_full + 2;               // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = a.nq / a.nkv;
  const int qb = blockIdx.x % a.q_blocks, hg = blockIdx.x / a.q_blocks;
  const int kvh = blockIdx.y, obs = blockIdx.z;
  const int head0 = kvh * group + hg * a.heads_per_cta;
  const int n_heads = min(a.heads_per_cta, group - hg * a.heads_per_cta);  // the last CTA may hold fewer
  // keys this CTA can see: up to the larger of causal_from - 1 and its last query's diagonal
  const int last_pos = a.heads_per_cta == 1 ? min(a.Lq, (qb + 1) * NG * kGqRows) - 1 : a.Lq - 1;
  long long last_key = a.causal_from - 1;
  if (last_pos + a.q_offset > last_key) last_key = last_pos + a.q_offset;
  if (last_key > a.Lk - 1) last_key = a.Lk - 1;
  // 128-key tiles of cache keys [0, min(last_key + 1, own_from)) through the TMA rings, then (with
  // own rows this CTA can see) one 64-key tile of the own keys from shared memory
  const bool own = a.k_own != nullptr;
  const long long own_from = own ? a.own_from : a.Lk;
  const long long cache_end = last_key + 1 < own_from ? last_key + 1 : own_from;
  const int n_cache = static_cast<int>((cache_end + kGqKeys - 1) / kGqKeys);
  const bool own_tile = own && last_key >= own_from;
  const int n_tiles = n_cache + (own_tile ? 1 : 0);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 4 * NG);
    for (int i = 0; i < kGqStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      grid_dep_wait();
      const uint64_t keep = policy_evict_normal();
      const int x = kvh * kGqHd;
      const int yk = static_cast<int>(obs * a.k_rows), yv = static_cast<int>(obs * a.v_rows);
      for (int j = 0; j < n_cache; ++j) {
        const int st = j % kGqStages;
        const uint32_t back = static_cast<uint32_t>(j / kGqStages - 1) & 1u;
        if (j >= kGqStages && !mbar_wait(&k_empty[st], back, a.status)) break;
        mbar_arrive_expect_tx(&k_full[st], kGqTile);
        tma_load_2d(smem + kGqOffK + st * kGqTile, &tm_k, &k_full[st], x, yk + j * kGqKeys, keep);
        if (j >= kGqStages && !mbar_wait(&v_empty[st], back, a.status)) break;
        mbar_arrive_expect_tx(&v_full[st], kGqTile);
        tma_load_2d(smem + kGqOffV + st * kGqTile, &tm_v, &v_full[st], x, yv + j * kGqKeys, keep);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_attn(kGqKeys, 0);
      constexpr uint32_t ID_O = idesc_attn(kGqHd, 1);
      constexpr uint32_t ID_S_OWN = idesc_attn(kGqOwn, 0);
      // tile j: a cache tile from the K ring (N 128), or the own tile (j == n_cache: N 64, staged
      // with the queries, so no ring barrier)
      auto issue_s = [&](int j, int g) {
        const uint64_t qd = sw128_desc(smem_u32(smem + kGqOffQ + g * kGqTile));
        const bool mine = j == n_cache;
        const uint64_t kd = sw128_desc(smem_u32(smem + (mine ? Cfg::kOffOwnK : kGqOffK + (j % kGqStages) * kGqTile)));
#pragma unroll
        for (int k = 0; k < kGqHd / 16; ++k)
          mma_f16(tmem + kGqColS + g * kGqKeys, qd + 2 * k, kd + 2 * k, mine ? ID_S_OWN : ID_S, k > 0 ? 1u : 0u);
        mma_commit(&s_full[g]);
      };
      bool ok = mbar_wait(q_full, 0, a.status) && (n_cache == 0 || mbar_wait(&k_full[0], 0, a.status));
      if (ok) {
        tc_fence_after();
        for (int g = 0; g < NG; ++g) issue_s(0, g);
        if (n_cache > 0) mma_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j % kGqStages;
        const bool mine = j == n_cache;
        if (j + 1 < n_tiles) {
          const int sn = (j + 1) % kGqStages;
          const bool next_mine = j + 1 == n_cache;
          if (!next_mine) ok = mbar_wait(&k_full[sn], static_cast<uint32_t>((j + 1) / kGqStages) & 1u, a.status);
          for (int g = 0; g < NG && ok; ++g) {
            ok = mbar_wait(&s_free[g], j & 1u, a.status);
            if (ok) {
              tc_fence_after();
              issue_s(j + 1, g);
            }
          }
          if (!ok) break;
          if (!next_mine) mma_commit(&k_empty[sn]);
        }
        if (!mine && !mbar_wait(&v_full[st], static_cast<uint32_t>(j / kGqStages) & 1u, a.status)) break;
        const uint64_t vd = sw128_desc(smem_u32(smem + (mine ? Cfg::kOffOwnV : kGqOffV + st * kGqTile)));
        const int ksteps = (mine ? kGqOwn : kGqKeys) / 16;
        for (int g = 0; g < NG && ok; ++g) {
          ok = mbar_wait(&p_full[g], j & 1u, a.status);
          if (!ok) break;
          tc_fence_after();
          for (int k = 0; k < ksteps; ++k)
            mma_f16_ta(tmem + kGqColO + g * kGqHd, tmem + kGqColP + g * (kGqKeys / 2) + 8 * k,
                       vd + static_cast<uint64_t>(k) * (2048 >> 4), ID_O, (j > 0 || k > 0) ? 1u : 0u);
          mma_commit(&o_full[g]);
        }
        if (!mine) mma_commit(&v_empty[st]);
      }
    }
  } else {
    // ---------------- queries, then softmax: group g, row r of the CTA (its TMEM lane)
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int rl = quad * 32 + lane;  // TMEM lane = row within the group
    // the own keys (rotated) and values into their 64-row tiles, in the rings' layout, by the
    // softmax threads of group 0 (two key and four value pieces each, every load in flight
    // together); rows past the own rows zero (their probabilities are zero, and zero values keep
    // P V finite)
    auto stage_own = [&]() {
      if (g != 0) return;
      const int n_own = static_cast<int>(a.Lk - own_from);
      const __nv_bfloat16* ko = a.k_own + obs * a.b_own + static_cast<long long>(kvh) * kGqHd;
      const __nv_bfloat16* vo = a.v_own + obs * a.b_own + static_cast<long long>(kvh) * kGqHd;
      uint8_t* okt = smem + Cfg::kOffOwnK;
      uint8_t* ovt = smem + Cfg::kOffOwnV;
      static_assert(kGqOwn * 4 == 2 * 128 && kGqOwn * 8 == 4 * 128, "pieces per thread");
      uint4 kv[2][2], vv[4];
#pragma unroll
      for (int it = 0; it < 2; ++it) {  // keys: row r, chunks c and c + 4
        const int idx = rl + 128 * it, r = idx >> 2, c = idx & 3;
        const uint4* kr = reinterpret_cast<const uint4*>(ko + static_cast<long long>(r < n_own ? r : 0) * a.ld_own);
        kv[it][0] = r < n_own ? __ldg(kr + c) : make_uint4(0u, 0u, 0u, 0u);
        kv[it][1] = r < n_own ? __ldg(kr + c + 4) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int it = 0; it < 4; ++it) {  // values: row r, chunk c
        const int idx = rl + 128 * it, r = idx >> 3, c = idx & 7;
        vv[it] = r < n_own ? __ldg(reinterpret_cast<const uint4*>(vo + static_cast<long long>(r) * a.ld_own) + c)
                           : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int idx = rl + 128 * it, r = idx >> 2, c = idx & 3;
        uint4 o1 = make_uint4(0u, 0u, 0u, 0u), o2 = o1;
        if (r < n_own) gq_rotate(kv[it][0], kv[it][1], a.k_cos + r * 32 + 8 * c, a.k_sin + r * 32 + 8 * c, o1, o2);
        *reinterpret_cast<uint4*>(okt + r * 128 + ((c ^ (r & 7)) << 4)) = o1;
        *reinterpret_cast<uint4*>(okt + r * 128 + (((c + 4) ^ (r & 7)) << 4)) = o2;
      }
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int idx = rl + 128 * it, r = idx >> 3, c = idx & 7;
        *reinterpret_cast<uint4*>(ovt + r * 128 + ((c ^ (r & 7)) << 4)) = vv[it];
      }
    };
    const int r = g * kGqRows + rl;
    int head = 0, pos = 0;
    const bool live = gqa_row<NG>(a, r, head0, n_heads, qb, head, pos);
    grid_dep_wait();
    {
      // this row's 64 query values, rotated in fp32 and rounded to bf16, into the K-major
      // SWIZZLE_128B tile (row rl: 128 bytes, 16-byte chunk c at (c ^ (rl & 7)) * 16)
      uint8_t* qt = smem + kGqOffQ + g * kGqTile + rl * 128;
      uint4 out[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) out[c] = make_uint4(0u, 0u, 0u, 0u);
      if (live) {
        const __nv_bfloat16* qr = a.q + obs * a.bq + static_cast<long long>(pos) * a.ldq + head * kGqHd;
        uint4 u[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) u[c] = __ldg(reinterpret_cast<const uint4*>(qr) + c);
        if (a.cos) {
          const float* cs = a.cos + static_cast<long long>(pos) * 32;
          const float* sn = a.sin + static_cast<long long>(pos) * 32;
#pragma unroll
          for (int c = 0; c < 4; ++c) {  // chunk c: dims 8c..8c+7 (first half), chunk c + 4: partners
            const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&u[c]);
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u[c + 4]);
            const float4 ca = __ldg(reinterpret_cast<const float4*>(cs + 8 * c));
            const float4 cb = __ldg(reinterpret_cast<const float4*>(cs + 8 * c + 4));
            const float4 sa = __ldg(reinterpret_cast<const float4*>(sn + 8 * c));
            const float4 sb = __ldg(reinterpret_cast<const float4*>(sn + 8 * c + 4));
            const float cv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
            const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
            __nv_bfloat162* p1 = reinterpret_cast<__nv_bfloat162*>(&out[c]);
            __nv_bfloat162* p2 = reinterpret_cast<__nv_bfloat162*>(&out[c + 4]);
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
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) out[c] = u[c];
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(qt + ((c ^ (rl & 7)) << 4)) = out[c];
      if (own_tile) stage_own();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(q_full);
    }

    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_addr = lane_base + kGqColS + g * kGqKeys;
    const uint32_t p_addr = lane_base + kGqColP + g * (kGqKeys / 2);
    const uint32_t o_addr = lane_base + kGqColO + g * kGqHd;
    const float sc = a.scale_log2;
    // keys [0, vis_end) are visible to this row (padding rows see key 0 only, and are dropped)
    long long vis_end = live ? pos + a.q_offset + 1 : 1;
    if (vis_end < a.causal_from) vis_end = a.causal_from;
    if (vis_end > a.Lk) vis_end = a.Lk;
    // visible keys of the cache tiles (below own_from) and of the own tile
    const int vis_cache = static_cast<int>(vis_end < own_from ? vis_end : own_from);
    const int vis_own = static_cast<int>(min(max(vis_end - own_from, 0LL), static_cast<long long>(kGqKeys)));
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (!mbar_wait(&s_full[g], j & 1u, a.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[kGqKeys];
#pragma unroll
      for (int c = 0; c < kGqKeys; c += 32) tmem_ld32(s_addr + c, sv + c);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[g]);
      // mask: keys at or past vis_end get -inf, and in a cache tile the cache rows of the own keys
      // (the own tile's column e is key own_from + e)
      const int nvis = j == n_cache ? vis_own : min(max(vis_cache - j * kGqKeys, 0), kGqKeys);
      if (nvis < kGqKeys) {
#pragma unroll
        for (int e = 0; e < kGqKeys; ++e)
          if (e >= nvis) sv[e] = __float_as_uint(-INFINITY);
      }
      float mx[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mx[t] = __uint_as_float(sv[t]);
#pragma unroll
      for (int e = 8; e < kGqKeys; e += 8)
#pragma unroll
        for (int t = 0; t < 8; ++t) mx[t] = fmaxf(mx[t], __uint_as_float(sv[e + t]));
      const float m_tile =
          fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sc;
      const bool raise = m_tile > m + kGqStaleMax;
      const float alpha = raise ? ex2(m - m_tile) : 1.f;
      if (raise) m = m_tile;
      // a fully masked tile (m_tile = -inf) keeps m; a row has seen key 0 before any such tile
      const float neg_m = m == -INFINITY ? 0.f : -m;
      uint32_t pk[kGqKeys / 2];
      float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < kGqKeys; e += 2) {
        float x0, x1;
        fma2(x0, x1, __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), sc, neg_m);
        const float p0 = ex2(x0), p1 = ex2(x1);
        const int t = (e >> 1) & 3;
        add2(ls[2 * t], ls[2 * t + 1], p0, p1);
        pk[e >> 1] = bf16x2(p0, p1);
      }
      const float s0 = (ls[0] + ls[2]) + (ls[4] + ls[6]), s1 = (ls[1] + ls[3]) + (ls[5] + ls[7]);
      if (j > 0) {
        if (!mbar_wait(&o_full[g], (j - 1) & 1u, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < kGqKeys / 2; c += 16) tmem_st16(p_addr + c, pk + c);
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
#pragma unroll
        for (int c = 0; c < kGqHd; c += 32) {
          uint32_t ov[32];
          tmem_ld32(o_addr + c, ov);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st16(o_addr + c, ov);
          tmem_st16(o_addr + c + 16, ov + 16);
        }
      }
      l = l * alpha + (s0 + s1);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
    }
    if (ok && mbar_wait(&o_full[g], (n_tiles - 1) & 1u, a.status)) {
      tc_fence_after();
      uint32_t ov[kGqHd];
      tmem_ld32(o_addr, ov);
      tmem_ld32(o_addr + 32, ov + 32);
      tmem_ld_wait();
      if (live) {
        const float inv = 1.f / l;
        uint4* dst = reinterpret_cast<uint4*>(a.o + obs * a.bo + static_cast<long long>(pos) * a.ldo + head * kGqHd);
#pragma unroll
        for (int q = 0; q < kGqHd / 8; ++q) {
          const float* v = reinterpret_cast<const float*>(ov) + 8 * q;
          dst[q] = make_uint4(bf16x2(v[0] * inv, v[1] * inv), bf16x2(v[2] * inv, v[3] * inv),
                              bf16x2(v[4] * inv, v[5] * inv), bf16x2(v[6] * inv, v[7] * inv));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, Cfg::kCols);
}

namespace {

using GqEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

GqEncodeFn gq_encode() {
  static GqEncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<GqEncodeFn>(p);
    return static_cast<GqEncodeFn>(nullptr);
  }();
  return fn;
}

// 128-row x 64-column boxes over `rows` rows of `cols` bf16 columns, row stride ld elements.
int gq_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld) {
  GqEncodeFn enc = gq_encode();
  if (!enc) return SO101_ERR_DRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? SO101_OK
             : SO101_ERR_ARG;
}

}  // namespace

// How a problem maps onto CTAs: groups of 128 rows per CTA (NG), query heads stacked per CTA,
// CTAs per kv head (head_groups) and 128 NG-row query blocks per head.
struct GqPlan {
  int ng, heads_per_cta, head_groups, q_blocks;
};

GqPlan gqa_plan(long long Lq, int nq, int nkv) {
  GqPlan p;
  const int group = nq / nkv;
  p.ng = 1;
  const long long rows = static_cast<long long>(p.ng) * kGqRows;
  p.heads_per_cta = Lq <= rows ? static_cast<int>(rows / Lq) : 1;
  if (p.heads_per_cta > group) p.heads_per_cta = group;
  p.head_groups = (group + p.heads_per_cta - 1) / p.heads_per_cta;
  p.q_blocks = p.heads_per_cta > 1 ? 1 : static_cast<int>((Lq + rows - 1) / rows);
  return p;
}

// Whether the masked tcgen05 kernel serves this problem: head_dim 64, bf16 output, K/V rows of
// every observation at a whole number of rows apart, 16-byte aligned rows and bases, enough
// CTAs to fill the GPU (the mma.sync kernel splits keys over clusters when there are few).
bool attention_gqa_tc_eligible(const void* q, long long ldq, const void* k, long long ldk, const void* v,
                               long long ldv, const void* o, long long ldo, int o_type, long long Lq, long long Lk,
                               int nq, int nkv, int hd, const float* cos, long long bq, long long bk, long long bv,
                               long long bo, int batch, const void* k_own, const void* v_own, long long ld_own,
                               long long b_own, long long own_from, const float* k_cos, const float* k_sin) {
  if (hd != 64 || o_type != SO101_BF16 || nq % nkv || Lq < 1 || Lk < 1) return false;
  if (k_own) {  // own rows: at most one 64-key tile, rows and rotary tables read in 16-byte pieces
    const auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
    if (!v_own || !k_cos || !k_sin || own_from < 0 || own_from > Lk || Lk - own_from > kGqOwn) return false;
    if (!a16(k_own) || !a16(v_own) || !a16(k_cos) || !a16(k_sin) || (ld_own * 2) % 16 || (b_own * 2) % 16)
      return false;
  }
  if (bk % ldk || bv % ldv || bk / ldk < Lk || bv / ldv < Lk || (batch > 1 && (bq < Lq * ldq || bo < Lq * ldo)))
    return false;
  const auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (!al(q) || !al(k) || !al(v) || !al(o) || (ldq * 2) % 16 || (ldk * 2) % 16 || (ldv * 2) % 16 ||
      (ldo * 2) % 16 || (bq * 2) % 16 || (bo * 2) % 16)
    return false;
  if (cos && reinterpret_cast<uintptr_t>(cos) % 16) return false;
  const GqPlan pl = gqa_plan(Lq, nq, nkv);
  const long long ctas = static_cast<long long>(pl.q_blocks) * pl.head_groups * nkv * batch;
  return ctas >= 128 && batch <= 65535 && Lk * batch < (1LL << 31) / 2;
}

int attention_gqa_tc_launch(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                            void* o, long long ldo, long long Lq, long long Lk, int nq, int nkv,
                            long long causal_from, long long q_offset, const float* cos, const float* sin, int batch,
                            long long bq, long long bk, long long bv, long long bo, const void* k_own,
                            const void* v_own, long long ld_own, long long b_own, long long own_from,
                            const float* k_cos, const float* k_sin, cudaStream_t stream) {
  const GqPlan pl = gqa_plan(Lq, nq, nkv);
  CUtensorMap tk, tv;
  const long long k_rows = bk / ldk, v_rows = bv / ldv;
  int rc = gq_map(&tk, k, k_rows * batch, static_cast<long long>(nkv) * 64, ldk);
  if (!rc) rc = gq_map(&tv, v, v_rows * batch, static_cast<long long>(nkv) * 64, ldv);
  if (rc) return rc;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e =
        cudaFuncSetAttribute(attention_gqa_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, GqCfg<1>::kSmem);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  GqaArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.ldq = ldq;
  a.bq = bq;
  a.o = static_cast<__nv_bfloat16*>(o);
  a.ldo = ldo;
  a.bo = bo;
  a.Lq = static_cast<int>(Lq);
  a.Lk = static_cast<int>(Lk);
  a.nq = nq;
  a.nkv = nkv;
  a.heads_per_cta = pl.heads_per_cta;
  a.q_blocks = pl.q_blocks;
  a.k_rows = k_rows;
  a.v_rows = v_rows;
  a.causal_from = causal_from;
  a.q_offset = q_offset;
  a.cos = cos;
  a.sin = sin;
  a.scale_log2 = static_cast<float>(1.4426950408889634 / 8.0);
  a.status = status_ptr();
  a.k_own = static_cast<const __nv_bfloat16*>(k_own);
  a.v_own = static_cast<const __nv_bfloat16*>(v_own);
  a.ld_own = ld_own;
  a.b_own = b_own;
  a.own_from = k_own ? own_from : Lk;
  a.k_cos = k_cos;
  a.k_sin = k_sin;
  const dim3 grid(static_cast<unsigned>(pl.q_blocks * pl.head_groups), static_cast<unsigned>(nkv),
                  static_cast<unsigned>(batch));
  return launch_kernel(attention_gqa_tc_kernel<1>, grid, dim3(GqCfg<1>::kThreads), GqCfg<1>::kSmem, stream, tk, tv, a);
}

}  // namespace so101
