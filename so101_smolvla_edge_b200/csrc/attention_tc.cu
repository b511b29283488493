// Flash attention on tcgen05 for the unmasked, equal-length case (SigLIP: 1024 tokens per image,
// 12 heads of 64, no RoPE): the vision tower's dominant kernel at batch 64.
//
// Persistent: one CTA per SM loops over work items, an item being 256 query rows of one (image,
// head) as two groups of 128 (MMA M = 128). The queries sit in two buffers (the next item's land
// while this one runs), the K/V rings and the group barriers run on across items, the next item's
// first S is issued before this item's last P V, and an item's output is stored while the next
// item's scores are computed. Per 128-key tile j:
//   warp 0 (one thread)  TMA: Q once per item, then K_j and V_j into separate four-stage rings (a K
//                        stage frees as soon as S_j is computed, so keys stream several tiles ahead)
//   warp 1 (elected lane) S_g = Q_g K_j^T  (M 128, N 128, K 64)      -> TMEM S_g
//                        O_g += P_g V_j   (M 128, N 64,  K 128 keys) -> TMEM O_g, A operand P_g
//                                                                       read from TMEM
//   warps 2-5 / 6-9      softmax for group A / B, one thread per query row (its TMEM lane): the
//                        row's 128 scores come into registers once, S_g is handed back for the
//                        next tile's MMA, and P = exp2(s * scale - m) goes to TMEM as bf16 pairs.
// The output accumulator stays in TMEM across tiles. The running row maximum m is only raised
// (and O_g, l rescaled, in TMEM) when a tile's maximum exceeds it by more than 2^8; otherwise the
// stale maximum stays, P values stay <= 2^8, and O / l is unchanged because O and l share the
// reference maximum.
// K and Q are K-major operands (head dim contiguous); V is an MN-major operand (head dim
// contiguous along N, keys along K) straight from its TMA tile. Softmax in fp32 with exp2 on
// log2(e)/sqrt(d)-scaled scores, P rounded to bf16 for P V, row sums from the fp32 P.
#include "tc_attn.cuh"

namespace so101 {

struct AttnTcArgs {
  void* o;
  long long ldo;
  int o_type;
  float o_qinv;
  int L;            // tokens per image (queries = keys)
  int heads;
  int items;        // (L / 256) x heads x images work items
  float scale_log2;
  int* status;
};

constexpr int kTcRows = 128;   // rows per group (MMA M)
constexpr int kTcKeys = 128;   // keys per tile (MMA N of S, K of P V)
constexpr int kTcHd = 64;
constexpr int kTcTile = kTcRows * kTcHd * 2;   // 16 KB: a 128 x 64 bf16 tile
constexpr int kTcThreads = 32 * (2 + 8);       // TMA warp, MMA warp, two softmax warp groups
constexpr float kStaleMax = 8.f;               // log2 of the largest factor a stale maximum allows
#ifndef SO101_ATTN_POLY_PAIRS
// batch 64, persistent kernel, two orders on one box: 904 / 911 us against 897 / 898 with 3
// (which moves the configs[0] W8A8 chunks outside the reference's own one-ulp band), 1018 with 1,
// 1030 with none; the non-persistent kernel measured 1049 with 2, 1087 with 4
#define SO101_ATTN_POLY_PAIRS 2
#endif
// Of every 16 score pairs, how many take exp2 from the polynomial (FMA pipe) instead of MUFU.
constexpr int kPolyPairs = SO101_ATTN_POLY_PAIRS;

// smem offsets (from a 1024-aligned base)
#ifndef SO101_ATTN_STAGES
#define SO101_ATTN_STAGES 4
#endif
constexpr int kStages = SO101_ATTN_STAGES;  // K and V ring depth (16 KB per stage each)
constexpr int kOffQ = 0;                              // 2 buffers x 2 groups x 16 KB
constexpr int kOffK = kOffQ + 4 * kTcTile;            // kStages x 16 KB
constexpr int kOffV = kOffK + kStages * kTcTile;      // kStages x 16 KB
constexpr int kOffBar = kOffV + kStages * kTcTile;
constexpr int kBarBytes = 512;  // 4 Q-buffer barriers, 4 x kStages ring barriers, 10 group barriers, TMEM slot
static_assert((4 + 4 * kStages + 10) * 8 + 4 <= kBarBytes, "barrier region");
constexpr int kTcSmem = kOffBar + kBarBytes + 1024;
static_assert(kTcSmem <= 232448, "227 KB of shared memory per CTA");

// TMEM columns: S_A, S_B (128 fp32 each), P_A, P_B (64 each: 128 bf16 keys in pairs), O_A, O_B (64)
constexpr uint32_t kColS = 0, kColP = 256, kColO = 384;

// 2^x for a pair, on the FMA and integer pipes instead of the MUFU unit (which the exp2 of the
// other pairs keeps busy). x = j + f with j = rint(x) and |f| <= 1/2: adding 1.5 * 2^23 rounds x
// to an integer held in the low mantissa bits of t; 2^f comes from a degree-3 polynomial (a
// relative-error minimax fit on [-1/2, 1/2] made for this kernel, max relative error 7.5e-5, far
// below the bf16 rounding P gets), and 2^j is added into its exponent field as (bits(t) << 23),
// whose low bits are j. x is clamped to >= -126 so the exponent cannot wrap.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = fadd2(x, make_float2(kRound, kRound));
  const float2 r = fadd2(t, make_float2(-kRound, -kRound));
  const float2 f = fadd2(x, make_float2(-r.x, -r.y));
  float2 q = ffma2(make_float2(5.517161265e-02f, 5.517161265e-02f), f, make_float2(2.426111251e-01f, 2.426111251e-01f));
  q = ffma2(q, f, make_float2(6.932609677e-01f, 6.932609677e-01f));
  q = ffma2(q, f, make_float2(9.999280572e-01f, 9.999280572e-01f));
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar;                       // [2] per Q buffer: the item's queries landed
  uint64_t* q_empty = q_full + 2;               // [2] per Q buffer: the item's S MMAs have read them
  uint64_t* k_full = q_empty + 2;               // [kStages]
  uint64_t* k_empty = k_full + kStages;         // [kStages]
  uint64_t* v_full = k_empty + kStages;         // [kStages]
  uint64_t* v_empty = v_full + kStages;         // [kStages]
  uint64_t* s_full = v_empty + kStages;         // [2] per group: S_g written
  uint64_t* s_free = s_full + 2;                // [2] per group: S_g read into registers
  uint64_t* p_full = s_free + 2;                // [2] per group: P_g written (and O_g rescaled)
  uint64_t* o_full = p_full + 2;                // [2] per group: P_g V accumulated into O_g
  uint64_t* o_free = o_full + 2;                // [2] per group: the item's O_g read out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = a.L / kTcKeys;
  const int qblocks = a.L / (2 * kTcRows);
  // work item w: query block w % qblocks of head (w / qblocks) % heads of image w / (qblocks * heads)
  auto item_rows = [&](int w, int& row0, int& key0, int& head) {
    const int img = w / (qblocks * a.heads);
    head = (w / qblocks) % a.heads;
    key0 = img * a.L;
    row0 = key0 + (w % qblocks) * 2 * kTcRows;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < kStages; ++i) {
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
      mbar_init(&o_free[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_launch();

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      grid_dep_wait();
      // Q is read once; K and V are read by the L / 256 items of this (image, head), which
      // neighbouring CTAs run at the same time, so they need no protection beyond the normal policy
      const uint64_t once = policy_evict_first(), keep = policy_evict_normal();
      bool ok = true;
      int t = 0;  // this CTA's key tile counter over all its items (ring slot and phase)
      for (int w = blockIdx.x, it = 0; w < a.items && ok; w += gridDim.x, ++it) {
        int row0, key0, head;
        item_rows(w, row0, key0, head);
        const int xq = head * kTcHd;
        const int qb = it & 1;
        if (it >= 2 && !mbar_wait(&q_empty[qb], static_cast<uint32_t>((it >> 1) - 1) & 1u, a.status)) break;
        mbar_arrive_expect_tx(&q_full[qb], 2 * kTcTile);
        tma_load_2d(smem + kOffQ + 2 * qb * kTcTile, &tm_q, &q_full[qb], xq, row0, once);
        tma_load_2d(smem + kOffQ + (2 * qb + 1) * kTcTile, &tm_q, &q_full[qb], xq, row0 + kTcRows, once);
        for (int j = 0; j < n_tiles; ++j, ++t) {
          const int st = t % kStages;
          const uint32_t back = static_cast<uint32_t>(t / kStages - 1) & 1u;  // phase of the use kStages ago
          if (t >= kStages && !mbar_wait(&k_empty[st], back, a.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], kTcTile);
          tma_load_2d(smem + kOffK + st * kTcTile, &tm_k, &k_full[st], xq, key0 + j * kTcKeys, keep);
          if (t >= kStages && !mbar_wait(&v_empty[st], back, a.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], kTcTile);
          tma_load_2d(smem + kOffV + st * kTcTile, &tm_v, &v_full[st], xq, key0 + j * kTcKeys, keep);
        }
      }
    }
  } else if (warp == 1) {
    // MMA issue: the whole warp runs the waits (their outcomes made warp-uniform: a timeout in any
    // lane ends the loop), its elected lane issues the MMAs and commits. The tile sequence runs
    // across this CTA's items: the next tile's S (possibly the next item's first) is issued
    // before this tile's P V, so the tensor pipe never waits for an item boundary.
    constexpr uint32_t ID_S = idesc_attn(kTcKeys, 0);
    constexpr uint32_t ID_O = idesc_attn(kTcHd, 1);
    auto wait = [&](uint64_t* b, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(b, parity, a.status)); };
    // S_t(g) = Q_g K_t^T into TMEM S_g, for key tile t of the item whose queries sit in buffer qb;
    // the queries' buffer is released after the S of the item's last tile
    auto issue_s = [&](int t, int qb, bool last_of_item) {
      const uint64_t kd = sw128_desc(smem_u32(smem + kOffK + (t % kStages) * kTcTile));
      bool ok = true;
      for (int g = 0; g < 2 && ok; ++g) {
        ok = t == 0 || wait(&s_free[g], static_cast<uint32_t>(t - 1) & 1u);  // S_g of tile t - 1 read
        if (!ok) break;
        tc_fence_after();
        const uint64_t qd = sw128_desc(smem_u32(smem + kOffQ + (2 * qb + g) * kTcTile));
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < kTcHd / 16; ++k)
            mma_f16(tmem + kColS + g * kTcKeys, qd + 2 * k, kd + 2 * k, ID_S, k > 0 ? 1u : 0u);
          mma_commit(&s_full[g]);
        }
      }
      if (ok && elect_one()) {
        mma_commit(&k_empty[t % kStages]);  // the K stage is free once both groups' S MMAs read it
        if (last_of_item) mma_commit(&q_empty[qb]);
      }
      return ok;
    };
    int w = blockIdx.x, it = 0, j = 0, t = 0;
    bool ok = w < a.items && wait(&q_full[0], 0) && wait(&k_full[0], 0) && issue_s(0, 0, n_tiles == 1);
    while (ok) {
      // tile t = tile j of item it, whose S is issued: issue the next tile's S, then P_t V_t
      const bool item_end = j + 1 == n_tiles;
      const int w_next = item_end ? w + static_cast<int>(gridDim.x) : w;
      const int it_next = item_end ? it + 1 : it;
      const int j_next = item_end ? 0 : j + 1;
      const bool more = w_next < a.items;
      if (more) {
        ok = (!item_end || wait(&q_full[it_next & 1], static_cast<uint32_t>(it_next >> 1) & 1u)) &&
             wait(&k_full[(t + 1) % kStages], static_cast<uint32_t>((t + 1) / kStages) & 1u) &&
             issue_s(t + 1, it_next & 1, j_next + 1 == n_tiles);
        if (!ok) break;
      }
      const int st = t % kStages;
      if (!wait(&v_full[st], static_cast<uint32_t>(t / kStages) & 1u)) break;
      const uint64_t vd = sw128_desc(smem_u32(smem + kOffV + st * kTcTile));
      for (int g = 0; g < 2 && ok; ++g) {
        // P_t written; on an item's first tile also the previous item's O_g read out (this P V
        // starts O_g afresh)
        ok = wait(&p_full[g], static_cast<uint32_t>(t) & 1u) &&
             (j > 0 || it == 0 || wait(&o_free[g], static_cast<uint32_t>(it - 1) & 1u));
        if (!ok) break;
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int k = 0; k < kTcKeys / 16; ++k)  // 16 keys = 8 P columns; V: 16 key rows = 2048 bytes
            mma_f16_ta(tmem + kColO + g * kTcHd, tmem + kColP + g * (kTcKeys / 2) + 8 * k,
                       vd + static_cast<uint64_t>(k) * (2048 >> 4), ID_O, (j > 0 || k > 0) ? 1u : 0u);
          mma_commit(&o_full[g]);
        }
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&v_empty[st]);
      if (!more) break;
      w = w_next, it = it_next, j = j_next, ++t;
    }
  } else {
    // ---------------- softmax: group g = (warp - 2) / 4, row r = quad * 32 + lane
    grid_dep_wait();
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_addr = lane_base + kColS + g * kTcKeys;
    const uint32_t p_addr = lane_base + kColP + g * (kTcKeys / 2);
    const uint32_t o_addr = lane_base + kColO + g * kTcHd;
    const float sc = a.scale_log2;
    bool ok = true;
    int t = 0;  // key tile counter over this CTA's items (the group barriers' phases)
    for (int w = blockIdx.x; w < a.items && ok; w += gridDim.x) {
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n_tiles; ++j, ++t) {
        if (!mbar_wait(&s_full[g], static_cast<uint32_t>(t) & 1u, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[kTcKeys];
#pragma unroll
        for (int c = 0; c < kTcKeys; c += 32) tmem_ld32(s_addr + c, sv + c);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[g]);  // the MMA may write the next tile's S now
        // row maximum over eight independent chains (short dependency chains keep the pipe busy)
        float mx[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = __uint_as_float(sv[e]);
#pragma unroll
        for (int e = 8; e < kTcKeys; e += 8)
#pragma unroll
          for (int c = 0; c < 8; ++c) mx[c] = fmaxf(mx[c], __uint_as_float(sv[e + c]));
        const float m_tile =
            fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sc;
        const bool raise = m_tile > m + kStaleMax;
        const float alpha = raise ? ex2(m - m_tile) : 1.f;  // 0 on an item's first tile (m = -inf)
        if (raise) m = m_tile;
        const float neg_m = -m;
        // P = exp2(s * scale - m) as bf16 pairs, in registers first: the previous tile's P V may
        // still be reading P_g, and it runs while these exponentials are computed
        uint32_t pk[kTcKeys / 2];
        float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // row sum over four packed chains
#pragma unroll
        for (int e = 0; e < kTcKeys; e += 2) {
          float x0, x1;
          fma2(x0, x1, __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]), sc, neg_m);
          float p0, p1;
          if (((e >> 1) & 15) < kPolyPairs) {
            const float2 pp = exp2_poly2(make_float2(x0, x1));
            p0 = pp.x, p1 = pp.y;
          } else {
            p0 = ex2(x0), p1 = ex2(x1);
          }
          const int c = (e >> 1) & 3;
          add2(ls[2 * c], ls[2 * c + 1], p0, p1);
          pk[e >> 1] = bf16x2(p0, p1);
        }
        const float s0 = (ls[0] + ls[2]) + (ls[4] + ls[6]), s1 = (ls[1] + ls[3]) + (ls[5] + ls[7]);
        if (j > 0) {
          // P_{t-1} V has landed: P_g may be overwritten and O_g is stable for a rescale (on an
          // item's first tile the previous item's read-out already waited for it)
          if (!mbar_wait(&o_full[g], static_cast<uint32_t>(t - 1) & 1u, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < kTcKeys / 2; c += 16) tmem_st16(p_addr + c, pk + c);
        if (j > 0 && __any_sync(0xffffffffu, raise)) {
          // the row maximum rose by more than 2^8 somewhere in this warp: rescale O_g rows
#pragma unroll
          for (int c = 0; c < kTcHd; c += 32) {
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
      // O / l for this row: read O_g out, hand it back to the MMA (the next item's first P V
      // overwrites it), then store while the next item's scores are computed
      if (!ok || !mbar_wait(&o_full[g], static_cast<uint32_t>(t - 1) & 1u, a.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t ov[kTcHd];
      tmem_ld32(o_addr, ov);
      tmem_ld32(o_addr + 32, ov + 32);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[g]);
      int row0, key0, head;
      item_rows(w, row0, key0, head);
      const float inv = 1.f / l;
      const long long orow = row0 + g * kTcRows + r;
      if (a.o_type == SO101_BF16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.o) + orow * a.ldo + head * kTcHd);
#pragma unroll
        for (int q = 0; q < kTcHd / 8; ++q) {
          const float* v = reinterpret_cast<const float*>(ov) + 8 * q;
          dst[q] = make_uint4(bf16x2(v[0] * inv, v[1] * inv), bf16x2(v[2] * inv, v[3] * inv),
                              bf16x2(v[4] * inv, v[5] * inv), bf16x2(v[6] * inv, v[7] * inv));
        }
      } else {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<int8_t*>(a.o) + orow * a.ldo + head * kTcHd);
#pragma unroll
        for (int q = 0; q < kTcHd / 16; ++q) {
          const float* v = reinterpret_cast<const float*>(ov) + 16 * q;
          dst[q] = make_uint4(pack4_i8(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv, a.o_qinv),
                              pack4_i8(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv, a.o_qinv),
                              pack4_i8(v[8] * inv, v[9] * inv, v[10] * inv, v[11] * inv, a.o_qinv),
                              pack4_i8(v[12] * inv, v[13] * inv, v[14] * inv, v[15] * inv, a.o_qinv));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// rows x 64-column boxes over a bf16 matrix of `rows` rows with row stride ld elements; the map's
// inner extent stops at `cols` so a box never reads past the head it starts in.
int map_rows(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld) {
  EncodeFn enc = encode();
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

// Whether the tcgen05 kernel serves this problem, and its launch.
bool attention_tc_eligible(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                           long long Lq, long long Lk, int nq, int nkv, int hd, long long causal_from,
                           const float* cos, long long bq, long long bk, long long bv, int o_type) {
  return hd == 64 && nq == nkv && Lq == Lk && Lq % 256 == 0 && causal_from >= Lk && !cos && bq == Lq * ldq &&
         bk == Lk * ldk && bv == Lk * ldv && (ldq * 2) % 16 == 0 && (ldk * 2) % 16 == 0 && (ldv * 2) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(v) % 16 == 0 && (o_type == SO101_BF16 || o_type == SO101_I8);
}

int attention_tc_launch(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                        void* o, long long ldo, int o_type, float o_qscale, long long L, int heads, int batch,
                        cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  const long long rows = L * batch, cols = static_cast<long long>(heads) * 64;
  int rc = map_rows(&tq, q, rows, cols, ldq);
  if (!rc) rc = map_rows(&tk, k, rows, cols, ldk);
  if (!rc) rc = map_rows(&tv, v, rows, cols, ldv);
  if (rc) return rc;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  AttnTcArgs a;
  a.o = o;
  a.ldo = ldo;
  a.o_type = o_type;
  a.o_qinv = o_type == SO101_I8 ? static_cast<float>(1.0 / static_cast<double>(o_qscale)) : 0.f;
  a.L = static_cast<int>(L);
  a.heads = heads;
  a.items = static_cast<int>(L / 256) * heads * batch;
  a.scale_log2 = static_cast<float>(1.4426950408889634 / 8.0);
  a.status = status_ptr();
  // persistent: one CTA per SM (TMEM and shared memory allow no more), each looping over items
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 148;
  }
  const int grid = a.items < sms ? a.items : sms;
  return launch_kernel(attention_tc_kernel, dim3(static_cast<unsigned>(grid)), dim3(kTcThreads), kTcSmem, stream,
                       tq, tk, tv, a);
}

}  // namespace so101
