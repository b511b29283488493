// The action expert's 16 layers of one denoising step as one persistent cooperative kernel, for a
// single observation (the 50 action rows): the batch-1 latency path.
//
// Launched with one CTA per SM (cooperative launch: every CTA is resident, so grid barriers and
// waits on other CTAs are safe). Per layer five phases, each separated by a grid barrier:
//   1  h = RMSNorm(e) * ln_in (built per CTA into the MMA's token operand), [q | k | v] = h W^T
//      (self layers; cross layers: q only); the epilogue rotates k (RoPE) and writes k, v into the
//      layer's cache rows [prefix_len, prefix_len + rows)
//   2  attention, one CTA per query head (mma.sync flash attention of attention_tile.cuh)
//   3  e += attn W_o^T
//   4  h = RMSNorm(e) * ln_post, act = silu(h W_gate^T) * (h W_up^T)
//   5  e += act W_down^T
// The GEMMs are the skinny-M weight-streaming kind: weights on the MMA M side (128 rows per tile,
// TMA, SWIZZLE_128B), the rows on MMA N (64, zero beyond `rows`), K split into work items of a few
// 64-wide blocks. Every item stores its fp32 partial, counts itself in the tile's ticket, waits
// until all of the tile's splits have stored theirs, then sums, in split order, the partials of
// its own slice of token columns and runs the epilogue for that slice: deterministic, and the
// reduction and epilogue of a tile run on all of its split CTAs at once. A CTA issues the TMA for
// the weights of its next GEMM item before it enters the barrier, so weight streaming overlaps the
// barrier and the phase in between; only the token operand waits. RMSNorm statistics travel as
// per-tile sums of squares written by the residual epilogues (phase 0 computes them for the
// step's input).
// Every wait is bounded; a timeout records SO101_ERR_TIMEOUT, raises an abort flag that releases
// every other waiter, and the kernel unwinds.
#include <mutex>

#include "attention_tile.cuh"

namespace so101 {

constexpr int kXsLayers = 16;
constexpr int kXsThreads = 128;
constexpr int kXsMaxKb = 4;                    // 64-wide K blocks per work item
constexpr int kXsWBlk = 128 * 64 * 2;          // one 128 x 64 bf16 weight block
constexpr int kXsBBlk = 64 * 64 * 2;           // one 64 x 64 bf16 token block
constexpr int kXsOffW = 0;                     // weights: gate/plain blocks, then up blocks
constexpr int kXsOffB = kXsOffW + 2 * kXsMaxKb * kXsWBlk;
constexpr int kXsOffStage = kXsOffB + kXsMaxKb * kXsBBlk;   // fp32 128 x 64 epilogue exchange
constexpr int kXsOffMisc = kXsOffStage + 128 * 64 * 4;
constexpr int kXsSmem = kXsOffMisc + 2048 + 1024;
constexpr int kXsGroup = 16;                   // CTAs per first-level barrier group
constexpr int kXsMaxGemmPhases = 4 * kXsLayers;
constexpr int kXsMaxTiles = 64;                // output tiles per GEMM (tickets per phase)
static_assert(kXsOffMisc - kXsOffB >= attention_smem_bytes<64>(), "attention reuses the token and stage areas");

enum XsGemmKind { kXsAttnIn = 0, kXsO = 1, kXsGateUp = 2, kXsDown = 3 };

struct XsLayer {
  const float* ln_in;
  const float* ln_post;
  __nv_bfloat16* k;  // self: key cache (prefix_len + rows rows), cross: expert keys (prefix_len rows)
  __nv_bfloat16* v;
  int self_attn;
};

struct XsParams {
  CUtensorMap maps[kXsLayers][4];  // per layer: attention-in (qkv or q), o, gate_up, down
  CUtensorMap tm_attn;             // token operand of o: attention output, rows x q_dim bf16
  CUtensorMap tm_act;              // token operand of down: SwiGLU output, rows x mlp_dim bf16
  XsLayer layer[kXsLayers];
  float* e;
  __nv_bfloat16* q;
  __nv_bfloat16* attn;
  __nv_bfloat16* act;
  float* partials;
  int* tickets;    // [GEMM phase][tile] arrivals
  unsigned* bar;   // [0] generation, [1] abort, [2] top count, [16 + g] group counts
  float* ss;       // per residual tile: sums of squares of e over the tile's columns, [tile][64]
  const float* cos_s;
  const float* sin_s;
  const float* cos_c;
  const float* sin_c;
  int n_layers, H, L, D, QD, KV, F, nq, nkv;
  int kbs[4];      // K blocks per work item, per GEMM kind
  float eps, scale_log2;
  int* status;
  unsigned long long wait_ns;  // bound of the grid-barrier and split-count waits
  int withhold;                // test hook: this CTA never arrives at a grid barrier (-1: none)
};

// ------------------------------------------------------------------------------ small helpers
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void xs_fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t xs_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Thread 0: wait (bounded, abort-aware) until *word >= target. Returns false on abort or timeout.
__device__ bool xs_wait_count(const XsParams& p, const unsigned* word, unsigned target) {
  const unsigned* abort = p.bar + 1;
  const uint64_t t0 = globaltimer();
  while (ld_acquire_u32(word) < target) {
    __nanosleep(64);
    if (ld_relaxed_u32(abort)) return false;
    if (globaltimer() - t0 > p.wait_ns) {
      record_error(p.status, SO101_ERR_TIMEOUT);
      atomicExch(const_cast<unsigned*>(abort), 1u);
      return false;
    }
  }
  return true;
}

// Grid-wide barrier in two levels: CTAs count in groups of kXsGroup, the last of each group counts
// in the top counter, and the last group resets the top count and advances the generation (the
// last arriver of each level resets that level's counter before it passes on, and nobody arrives
// again before the generation moves). Waiters poll the generation with a short back-off. A CTA
// that arrives with ok == false raises the abort flag; waiters give up on abort or after the wait
// limit (recording SO101_ERR_TIMEOUT). Returns whether every CTA is still good.
__device__ bool xs_grid_sync(const XsParams& p, bool ok, int* s_flag) {
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && static_cast<int>(blockIdx.x) == p.withhold) {
    // test hook: leave without arriving (and without raising the abort flag), so that every
    // other CTA's wait runs into its bound
    *s_flag = 0;
  } else if (threadIdx.x == 0) {
    unsigned* gen = p.bar;
    unsigned* abort = p.bar + 1;
    unsigned* top = p.bar + 2;
    if (!ok) atomicExch(abort, 1u);
    int good = ok && ld_relaxed_u32(abort) == 0;
    const unsigned g = ld_acquire_u32(gen);
    __threadfence();
    const unsigned grp = blockIdx.x / kXsGroup;
    const unsigned ngrp = (gridDim.x + kXsGroup - 1) / kXsGroup;
    const unsigned gsize = min(static_cast<unsigned>(kXsGroup), gridDim.x - grp * kXsGroup);
    bool released = false;
    if (atomicAdd(p.bar + 16 + grp, 1u) == gsize - 1) {
      atomicExch(p.bar + 16 + grp, 0u);
      __threadfence();
      if (atomicAdd(top, 1u) == ngrp - 1) {
        atomicExch(top, 0u);
        __threadfence();
        atomicAdd(gen, 1u);
        released = true;
      }
    }
    if (!released) {
      const uint64_t t0 = globaltimer();
      while (ld_acquire_u32(gen) == g) {
        __nanosleep(100);
        if (ld_relaxed_u32(abort)) {
          good = 0;
          break;
        }
        if (globaltimer() - t0 > p.wait_ns) {
          record_error(p.status, SO101_ERR_TIMEOUT);
          atomicExch(abort, 1u);
          good = 0;
          break;
        }
      }
    }
    __threadfence();
    if (ld_relaxed_u32(abort)) good = 0;
    *s_flag = good;
  }
  __syncthreads();
  tc_fence_after();
  return *s_flag != 0;
}

// ------------------------------------------------------------------------------ GEMM items
struct XsGemm {
  const CUtensorMap* map;
  int n, k, tiles, kb, kbs, splits, dual;
};

__device__ __forceinline__ XsGemm xs_gemm(const XsParams& p, int layer, int kind) {
  XsGemm g;
  g.map = &p.maps[layer][kind];
  g.dual = kind == kXsGateUp;
  switch (kind) {
    case kXsAttnIn:
      g.n = p.QD + (p.layer[layer].self_attn ? 2 * p.KV : 0);
      g.k = p.D;
      break;
    case kXsO:
      g.n = p.D;
      g.k = p.QD;
      break;
    case kXsGateUp:
      g.n = p.F;
      g.k = p.D;
      break;
    default:
      g.n = p.D;
      g.k = p.F;
      break;
  }
  g.tiles = (g.n + 127) / 128;
  g.kb = (g.k + 63) / 64;
  g.kbs = p.kbs[kind];
  g.splits = (g.kb + g.kbs - 1) / g.kbs;
  return g;
}

struct XsState {
  uint8_t* smem;
  uint64_t* wbar;   // weights TMA
  uint64_t* bbar;   // token operand TMA
  uint64_t* mbar;   // MMA completion
  float* rstd;      // [64]
  float* red;       // [4][64]
  int* flag;
  uint32_t tmem;
  int w_issued, w_waited, b_waited, m_waited;
  int gphase;                 // GEMM phases so far (the ticket row)
  int pref_layer, pref_kind;  // weights already in flight for item blockIdx.x of this GEMM
  bool ok;
};

// Thread 0: TMA of the weight blocks of one item (gate and up tiles for the SwiGLU GEMM).
__device__ void xs_load_w(const XsParams& p, XsState& st, const XsGemm& g, int item) {
  const int t = item / g.splits, s = item % g.splits;
  const int kb0 = s * g.kbs, kbn = min(g.kbs, g.kb - kb0);
  mbar_arrive_expect_tx(st.wbar, kbn * kXsWBlk * (g.dual ? 2 : 1));
  const uint64_t pol = policy_evict_first();
  for (int i = 0; i < kbn; ++i) {
    tma_load_2d(st.smem + kXsOffW + i * kXsWBlk, g.map, st.wbar, (kb0 + i) * 64, t * 128, pol);
    if (g.dual)
      tma_load_2d(st.smem + kXsOffW + (kXsMaxKb + i) * kXsWBlk, g.map, st.wbar, (kb0 + i) * 64, p.F + t * 128, pol);
  }
  ++st.w_issued;
}

// Before a barrier: start the weights of this CTA's first item of the next GEMM.
__device__ void xs_prefetch(const XsParams& p, XsState& st, int layer, int kind) {
  if (layer >= p.n_layers) return;
  const XsGemm g = xs_gemm(p, layer, kind);
  if (static_cast<int>(blockIdx.x) >= g.tiles * g.splits) return;
  if (threadIdx.x == 0) xs_load_w(p, st, g, blockIdx.x);
  st.pref_layer = layer;
  st.pref_kind = kind;
}

// RMSNorm token operand: K blocks [kb0, kb0 + kbn) of bf16((e * rstd) * w), SWIZZLE_128B K-major
// (64 rows x 64 k per block), zero beyond `rows` and beyond K. Loads in batches of eight 16-byte
// chunks per thread, all issued before any is used.
__device__ void xs_build_b_norm(const XsParams& p, const XsState& st, int kb0, int kbn, int K,
                                const float* __restrict__ w_ln) {
  uint8_t* b = st.smem + kXsOffB;
  const int chunks = kbn * 512;
  for (int base = 0; base < chunks; base += 8 * kXsThreads) {
    float4 x0[8], x1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = base + i * kXsThreads + threadIdx.x;
      const int blk = c >> 9, m = (c >> 3) & 63, ch = c & 7;
      const int k = (kb0 + blk) * 64 + ch * 8;
      x0[i] = x1[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < chunks && m < p.H && k < K) {
        const float* x = p.e + static_cast<long long>(m) * p.D + k;
        x0[i] = __ldcg(reinterpret_cast<const float4*>(x));
        x1[i] = __ldcg(reinterpret_cast<const float4*>(x + 4));
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = base + i * kXsThreads + threadIdx.x;
      if (c >= chunks) continue;
      const int blk = c >> 9, m = (c >> 3) & 63, ch = c & 7;
      const int k = (kb0 + blk) * 64 + ch * 8;
      uint4 out = make_uint4(0u, 0u, 0u, 0u);
      if (m < p.H && k < K) {
        const float4 w0 = *reinterpret_cast<const float4*>(w_ln + k);
        const float4 w1 = *reinterpret_cast<const float4*>(w_ln + k + 4);
        const float r = st.rstd[m];
        out = make_uint4(xs_bf16x2((x0[i].x * r) * w0.x, (x0[i].y * r) * w0.y),
                         xs_bf16x2((x0[i].z * r) * w0.z, (x0[i].w * r) * w0.w),
                         xs_bf16x2((x1[i].x * r) * w1.x, (x1[i].y * r) * w1.y),
                         xs_bf16x2((x1[i].z * r) * w1.z, (x1[i].w * r) * w1.w));
      }
      *reinterpret_cast<uint4*>(b + blk * kXsBBlk + (m >> 3) * 1024 + (m & 7) * 128 + ((ch ^ (m & 7)) << 4)) = out;
    }
  }
}

// rstd of every row from the residual tiles' sums of squares (summed in tile order).
__device__ void xs_rstd(const XsParams& p, XsState& st) {
  const int nt = (p.D + 127) / 128;
  if (threadIdx.x < 64) {
    float v[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) v[t] = t < nt ? __ldcg(p.ss + t * 64 + threadIdx.x) : 0.f;
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < 16; ++t) s += v[t];
    st.rstd[threadIdx.x] = rsqrtf(s / static_cast<float>(p.D) + p.eps);
  }
  __syncthreads();
}

enum XsEpi { kEpiQkv = 0, kEpiQ = 1, kEpiResid = 2, kEpiGate = 3 };

// Epilogue of this CTA's token-column slice [c0, c1) of tile t: the summed accumulators are in
// shared memory, stage[row][j] (and, for SwiGLU, upv[row][j]), j = m - c0. Loops run in batches
// of eight columns: compact code (the kernel runs each phase's code once per step, so straight-
// line unrolled code would mostly run from instruction-cache misses) with the loads of a batch in
// flight together.
__device__ void xs_epilogue(const XsParams& p, XsState& st, int layer, int epi, int t, int c0, int c1,
                            const float* stage, const float* upv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = threadIdx.x, n = t * 128 + row;
  const int cs = c1 - c0;
  if (epi == kEpiResid) {
    const bool live = n < p.D;
#pragma unroll 1
    for (int jb = 0; jb < cs; jb += 8) {
      float ev[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        ev[i] = (live && jb + i < cs) ? __ldcg(p.e + static_cast<long long>(c0 + jb + i) * p.D + n) : 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (live && jb + i < cs) {
          ev[i] += stage[row * 64 + jb + i];
          p.e[static_cast<long long>(c0 + jb + i) * p.D + n] = ev[i];
        }
        // this tile's sum of squares of the new e for column c0 + jb + i
        float sq = ev[i] * ev[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0 && jb + i < cs) st.red[warp * 64 + jb + i] = sq;
      }
    }
    __syncthreads();
    if (threadIdx.x < cs)
      p.ss[t * 64 + c0 + threadIdx.x] = (st.red[threadIdx.x] + st.red[64 + threadIdx.x]) +
                                        (st.red[128 + threadIdx.x] + st.red[192 + threadIdx.x]);
  } else if (epi == kEpiGate) {
    if (n < p.F) {
#pragma unroll 1
      for (int j = 0; j < cs; ++j)
        p.act[static_cast<long long>(c0 + j) * p.F + n] = __float2bfloat16_rn(silu(stage[row * 64 + j]) * upv[row * 64 + j]);
    }
  } else {
    // q | k | v: k needs its rotary partner row (32 rows away, same head); the stage holds every
    // row of the tile. Values are rounded to bf16 first (the q | k | v output precision).
    const XsLayer& ly = p.layer[layer];
    const int kv_end = p.QD + (ly.self_attn ? 2 * p.KV : 0);
    if (n >= kv_end) return;  // zero rows past the last weight row of the tile (cross layers: past q)
    if (n < p.QD) {
#pragma unroll 1
      for (int j = 0; j < cs; ++j)
        p.q[static_cast<long long>(c0 + j) * p.QD + n] = __float2bfloat16_rn(stage[row * 64 + j]);
    } else if (n < p.QD + p.KV) {
      const int c = n - p.QD, d = c & 63, half = 32;
      const int prow = d < half ? row + half : row - half;
      const int di = d & (half - 1);
#pragma unroll 1
      for (int j = 0; j < cs; ++j) {
        const int m = c0 + j;
        const float own = __bfloat162float(__float2bfloat16_rn(stage[row * 64 + j]));
        const float other = __bfloat162float(__float2bfloat16_rn(stage[prow * 64 + j]));
        const float cs_ = p.cos_s[m * half + di], sn = p.sin_s[m * half + di];
        const float r = d < half ? __fsub_rn(__fmul_rn(own, cs_), __fmul_rn(other, sn))
                                 : __fadd_rn(__fmul_rn(own, cs_), __fmul_rn(other, sn));
        ly.k[static_cast<long long>(p.L + m) * p.KV + c] = __float2bfloat16_rn(r);
      }
    } else {
      const int c = n - p.QD - p.KV;
#pragma unroll 1
      for (int j = 0; j < cs; ++j)
        ly.v[static_cast<long long>(p.L + c0 + j) * p.KV + c] = __float2bfloat16_rn(stage[row * 64 + j]);
    }
  }
}

// One GEMM phase: this CTA's items (item = blockIdx.x + i * gridDim.x). NORM: the token operand
// is RMSNorm(e) * w_ln, built here; otherwise `src_map` brings a bf16 matrix by TMA.
template <bool NORM>
__device__ void xs_gemm_phase(const XsParams& p, XsState& st, int layer, int kind, int epi, const float* w_ln,
                              const CUtensorMap* src_map) {
  const XsGemm g = xs_gemm(p, layer, kind);
  const int items = g.tiles * g.splits;
  int* tickets = p.tickets + st.gphase * kXsMaxTiles;
  ++st.gphase;
  if (static_cast<int>(blockIdx.x) >= items) return;
  if (NORM) xs_rstd(p, st);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cols = g.dual ? 128 : 64;
  // token-column slice per split: a multiple of 4 columns
  const int cs = ((p.H + g.splits - 1) / g.splits + 3) & ~3;
  for (int item = blockIdx.x; item < items && st.ok; item += gridDim.x) {
    const int t = item / g.splits, s = item % g.splits;
    const int kb0 = s * g.kbs, kbn = min(g.kbs, g.kb - kb0);
    const bool prefetched = item == static_cast<int>(blockIdx.x) && st.pref_layer == layer && st.pref_kind == kind;
    if (threadIdx.x == 0) {
      if (!prefetched) xs_load_w(p, st, g, item);
      if (!NORM) {
        mbar_arrive_expect_tx(st.bbar, kbn * kXsBBlk);
        for (int i = 0; i < kbn; ++i)
          tma_load_2d(st.smem + kXsOffB + i * kXsBBlk, src_map, st.bbar, (kb0 + i) * 64, 0, policy_evict_first());
      }
    }
    st.pref_layer = -1;
    if (NORM) {
      xs_build_b_norm(p, st, kb0, kbn, g.k, w_ln);
      xs_fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
      bool good = mbar_wait(st.wbar, static_cast<uint32_t>(st.w_waited) & 1u, p.status);
      if (!NORM) good = good && mbar_wait(st.bbar, static_cast<uint32_t>(st.b_waited) & 1u, p.status);
      if (good) {
        tc_fence_after();
        constexpr uint32_t idesc = idesc_bf16(128, 64);
        for (int i = 0; i < kbn; ++i) {
          const uint64_t ad = sw128_desc(smem_u32(st.smem + kXsOffW + i * kXsWBlk));
          const uint64_t bd = sw128_desc(smem_u32(st.smem + kXsOffB + i * kXsBBlk));
          const uint64_t ud = sw128_desc(smem_u32(st.smem + kXsOffW + (kXsMaxKb + i) * kXsWBlk));
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
            mma_f16(st.tmem, ad + 2 * k, bd + 2 * k, idesc, acc);
            if (g.dual) mma_f16(st.tmem + 64, ud + 2 * k, bd + 2 * k, idesc, acc);
          }
        }
        mma_commit(st.mbar);
      }
      *st.flag = good;
    }
    __syncthreads();
    ++st.w_waited;
    if (!NORM) ++st.b_waited;
    if (!*st.flag) {
      st.ok = false;
      break;
    }
    if (!mbar_wait(st.mbar, static_cast<uint32_t>(st.m_waited) & 1u, p.status)) st.ok = false;
    ++st.m_waited;
    if (__syncthreads_and(st.ok) == 0) {
      st.ok = false;
      break;
    }
    tc_fence_after();
    // accumulator row (weight row) = this thread's TMEM lane; the token operand area is free now
    const int row = warp * 32 + lane;
    const uint32_t taddr = st.tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float* stage = reinterpret_cast<float*>(st.smem + kXsOffStage);
    float* upv = reinterpret_cast<float*>(st.smem + kXsOffB);
    int c0 = 0, c1 = p.H;
    if (g.splits == 1) {
#pragma unroll 1
      for (int h = 0; h < (g.dual ? 2 : 1); ++h) {
        float* dst = h ? upv : stage;
#pragma unroll 1
        for (int c = 0; c < 64; c += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + h * 64 + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(dst + row * 64 + c + j) =
                make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
        }
      }
    } else {
      // store this split's partial
      float* part = p.partials + (static_cast<long long>(t * g.splits + s) * 128 + row) * cols;
#pragma unroll 1
      for (int c = 0; c < cols; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; j += 4)
          __stcg(reinterpret_cast<float4*>(part + c + j), make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                       __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])));
      }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        atomicAdd(tickets + t, 1);
        *st.flag = xs_wait_count(p, reinterpret_cast<const unsigned*>(tickets + t), static_cast<unsigned>(g.splits));
      }
      __syncthreads();
      if (!*st.flag) {
        st.ok = false;
        break;
      }
      __threadfence();
      // sum this split's token-column slice over every split, in split order (at most eight
      // splits' loads in flight at once, summed in order)
      c0 = s * cs;
      c1 = min(p.H, c0 + cs);
#pragma unroll 1
      for (int h = 0; h < (g.dual ? 2 : 1); ++h) {
        float* dst = h ? upv : stage;
#pragma unroll 1
        for (int j = 0; j < c1 - c0; j += 4) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
          for (int sb = 0; sb < g.splits; sb += 8) {
            float4 q4[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              q4[i] = sb + i < g.splits
                          ? __ldcg(reinterpret_cast<const float4*>(
                                p.partials + (static_cast<long long>(t * g.splits + sb + i) * 128 + row) * cols + h * 64 + c0 + j))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (sb + i < g.splits) acc.x += q4[i].x, acc.y += q4[i].y, acc.z += q4[i].z, acc.w += q4[i].w;
          }
          *reinterpret_cast<float4*>(dst + row * 64 + j) = acc;
        }
      }
    }
    __syncthreads();  // the QKV epilogue reads other rows' values
    if (c1 > c0) xs_epilogue(p, st, layer, epi, t, c0, c1, stage, upv);
    __syncthreads();  // the stage and reduction areas are reused by the next item
  }
}

// Attention phase: one item per query head.
__device__ void xs_attention_phase(const XsParams& p, XsState& st, int layer) {
  const XsLayer& ly = p.layer[layer];
  AttnArgs a;
  a.q = p.q;
  a.k = ly.k;
  a.v = ly.v;
  a.o = p.attn;
  a.ldq = p.QD;
  a.ldk = p.KV;
  a.ldv = p.KV;
  a.ldo = p.QD;
  a.bq = a.bk = a.bv = a.bo = 0;
  a.o_type = SO101_BF16;
  a.o_qscale = 0.f;
  a.Lq = p.H;
  a.Lk = ly.self_attn ? p.L + p.H : p.L;
  a.nq = p.nq;
  a.nkv = p.nkv;
  a.causal_from = p.L;
  a.q_offset = ly.self_attn ? p.L : 0;
  a.cos = ly.self_attn ? p.cos_s : p.cos_c;
  a.sin = ly.self_attn ? p.sin_s : p.sin_c;
  a.scale_log2 = p.scale_log2;
  a.kv_splits = 1;
  for (int h = blockIdx.x; h < p.nq; h += gridDim.x) {
    attention_body<64, false>(a, 0, 0, h, 0, st.smem + kXsOffB);
    __syncthreads();
  }
}

// Phase 0: sums of squares of the step's input e per residual tile.
__device__ void xs_ss_phase(const XsParams& p) {
  const int nt = (p.D + 127) / 128;
  for (int t = blockIdx.x; t < nt; t += gridDim.x) {
    if (threadIdx.x < 64) {
      float s = 0.f;
      const int m = threadIdx.x;
      if (m < p.H) {
        const int n_end = min(p.D, t * 128 + 128);
        for (int n = t * 128; n < n_end; ++n) {
          const float x = __ldcg(p.e + static_cast<long long>(m) * p.D + n);
          s += x * x;
        }
      }
      p.ss[t * 64 + m] = s;
    }
  }
}

__global__ void __launch_bounds__(kXsThreads, 1) expert_step_kernel(const __grid_constant__ XsParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  XsState st;
  st.smem = smem;
  st.wbar = reinterpret_cast<uint64_t*>(smem + kXsOffMisc);
  st.bbar = st.wbar + 1;
  st.mbar = st.wbar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(st.wbar + 3);
  st.flag = reinterpret_cast<int*>(st.wbar + 4);
  st.rstd = reinterpret_cast<float*>(smem + kXsOffMisc + 64);
  st.red = st.rstd + 64;
  st.w_issued = st.w_waited = st.b_waited = st.m_waited = 0;
  st.gphase = 0;
  st.pref_layer = st.pref_kind = -1;
  st.ok = true;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(st.wbar, 1);
    mbar_init(st.bbar, 1);
    mbar_init(st.mbar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_attn);
    tma_prefetch_desc(&p.tm_act);
    for (int l = 0; l < p.n_layers; ++l)
      for (int k = 0; k < 4; ++k) tma_prefetch_desc(&p.maps[l][k]);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  st.tmem = *tmem_slot;
  grid_dep_wait();

  xs_ss_phase(p);
  xs_prefetch(p, st, 0, kXsAttnIn);
  st.ok = xs_grid_sync(p, st.ok, st.flag);
  for (int l = 0; l < p.n_layers && st.ok; ++l) {
    const XsLayer& ly = p.layer[l];
    xs_gemm_phase<true>(p, st, l, kXsAttnIn, ly.self_attn ? kEpiQkv : kEpiQ, ly.ln_in, nullptr);
    xs_prefetch(p, st, l, kXsO);
    st.ok = xs_grid_sync(p, st.ok, st.flag);
    if (!st.ok) break;
    xs_attention_phase(p, st, l);
    st.ok = xs_grid_sync(p, st.ok, st.flag);
    if (!st.ok) break;
    xs_gemm_phase<false>(p, st, l, kXsO, kEpiResid, nullptr, &p.tm_attn);
    xs_prefetch(p, st, l, kXsGateUp);
    st.ok = xs_grid_sync(p, st.ok, st.flag);
    if (!st.ok) break;
    xs_gemm_phase<true>(p, st, l, kXsGateUp, kEpiGate, ly.ln_post, nullptr);
    xs_prefetch(p, st, l, kXsDown);
    st.ok = xs_grid_sync(p, st.ok, st.flag);
    if (!st.ok) break;
    xs_gemm_phase<false>(p, st, l, kXsDown, kEpiResid, nullptr, &p.tm_act);
    xs_prefetch(p, st, l + 1, kXsAttnIn);
    st.ok = xs_grid_sync(p, st.ok, st.flag);
  }
  // weights still in flight (an abort between prefetch and use): let them land before exit
  if (threadIdx.x == 0 && st.w_issued > st.w_waited)
    mbar_wait(st.wbar, static_cast<uint32_t>(st.w_waited) & 1u, p.status);
  grid_dep_launch();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(st.tmem, 128);
}

// ------------------------------------------------------------------------------ host
namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn xs_encode() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// rows x k bf16 matrix (row stride k), box_rows x 64-column boxes, SWIZZLE_128B.
int xs_map(CUtensorMap* m, const void* w, long long rows, long long k, unsigned box_rows = 128) {
  EncodeFn enc = xs_encode();
  if (!enc) return SO101_ERR_DRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? SO101_OK
             : SO101_ERR_ARG;
}

bool al16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

int xs_sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// K blocks per work item: enough items to spread over the GPU, at most six partials per tile.
int xs_kbs(int n, int k, int sms) {
  const int tiles = (n + 127) / 128, kb = (k + 63) / 64;
  int splits = sms / (2 * tiles);
  if (splits > 6) splits = 6;
  if (splits < 1) splits = 1;
  int kbs = (kb + splits - 1) / splits;
  if (kbs > kXsMaxKb) kbs = kXsMaxKb;
  return kbs;
}

// Test hooks (so101_expert_step_test_hooks): read at each launch, so they reach eager launches
// only; a CUDA graph keeps the values its capture saw.
long long g_xs_wait_ns = 0;  // 0: kWaitLimitNs
int g_xs_withhold = -1;

struct XsLayout {
  long long partials, tickets, bar, ss, total;
};

XsLayout xs_layout(const so101_expert_step* s, int sms) {
  long long most = 0;
  const int ns[4] = {s->q_dim + 2 * s->kv_dim, s->exp_dim, s->mlp_dim, s->exp_dim};
  const int ks[4] = {s->exp_dim, s->q_dim, s->exp_dim, s->mlp_dim};
  for (int i = 0; i < 4; ++i) {
    const int tiles = (ns[i] + 127) / 128, kb = (ks[i] + 63) / 64;
    const int kbs = xs_kbs(ns[i], ks[i], sms);
    const long long splits = (kb + kbs - 1) / kbs;
    const long long bytes = tiles * splits * 128LL * (i == kXsGateUp ? 128 : 64) * 4;
    if (bytes > most) most = bytes;
  }
  XsLayout l;
  l.partials = 0;
  l.tickets = (most + 255) / 256 * 256;
  l.bar = l.tickets + static_cast<long long>(kXsMaxGemmPhases) * kXsMaxTiles * 4;
  l.ss = l.bar + 256;
  l.total = l.ss + 16 * 64 * 4;
  return l;
}

int xs_check(const so101_expert_step* s) {
  if (!s || s->n_layers < 1 || s->n_layers > kXsLayers) return SO101_ERR_ARG;
  if (s->rows < 1 || s->rows > 64 || s->head_dim != 64 || s->prefix_len < 0) return SO101_ERR_ARG;
  if (s->n_kv < 1 || s->n_heads % s->n_kv || s->q_dim != s->n_heads * 64 || s->kv_dim != s->n_kv * 64)
    return SO101_ERR_ARG;
  if (s->exp_dim % 8 || s->mlp_dim % 8 || s->exp_dim > 16 * 128 || s->exp_dim < 8 || s->mlp_dim < 8) return SO101_ERR_ARG;
  // at most 64 output tiles per GEMM (the ticket array)
  if (s->q_dim + 2 * s->kv_dim > 64 * 128 || s->mlp_dim > 64 * 128) return SO101_ERR_ARG;
  if (!al16(s->e) || !al16(s->q) || !al16(s->attn) || !al16(s->act) || !al16(s->workspace) || !s->cos_self ||
      !s->sin_self || !s->cos_cross || !s->sin_cross)
    return SO101_ERR_ARG;
  for (int l = 0; l < s->n_layers; ++l) {
    const so101_expert_layer& y = s->layer[l];
    if (!y.w_attn || !y.w_o || !y.w_gate_up || !y.w_down || !y.ln_in || !y.ln_post || !y.k || !y.v) return SO101_ERR_ARG;
    if (!al16(y.w_attn) || !al16(y.w_o) || !al16(y.w_gate_up) || !al16(y.w_down) || !al16(y.ln_in) ||
        !al16(y.ln_post) || !al16(y.k) || !al16(y.v))
      return SO101_ERR_ARG;
  }
  return SO101_OK;
}

// Every work item of a GEMM gets its own CTA (a split waits for the other splits of its tile).
bool xs_items_fit(const so101_expert_step* s, int grid) {
  const int ns[4] = {s->q_dim + 2 * s->kv_dim, s->exp_dim, s->mlp_dim, s->exp_dim};
  const int ks[4] = {s->exp_dim, s->q_dim, s->exp_dim, s->mlp_dim};
  for (int i = 0; i < 4; ++i) {
    const int tiles = (ns[i] + 127) / 128, kb = (ks[i] + 63) / 64, kbs = xs_kbs(ns[i], ks[i], grid);
    if (tiles * ((kb + kbs - 1) / kbs) > grid) return false;
  }
  return true;
}

}  // namespace

}  // namespace so101

using namespace so101;

extern "C" int so101_expert_step_workspace(const so101_expert_step* s, int64_t* bytes) {
  if (!bytes) return SO101_ERR_ARG;
  const int rc = xs_check(s);
  if (rc) return rc;
  const int sms = xs_sms() < 256 ? xs_sms() : 256;
  if (!xs_items_fit(s, sms)) return SO101_ERR_ARG;
  *bytes = xs_layout(s, sms).total;
  return SO101_OK;
}

extern "C" int so101_expert_step_run(const so101_expert_step* s, cudaStream_t stream) {
  int rc = xs_check(s);
  if (rc) return rc;
  const int sms = xs_sms() < 256 ? xs_sms() : 256;  // 16 barrier groups of 16 at most
  if (!xs_items_fit(s, sms)) return SO101_ERR_ARG;
  const XsLayout lay = xs_layout(s, sms);
  if (s->workspace_bytes < lay.total) return SO101_ERR_WORKSPACE;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return SO101_ERR_LAUNCH;
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(expert_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kXsSmem);
    if (e != cudaSuccess) return launch_error(e);
    configured[dev] = true;
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, expert_step_kernel, kXsThreads, kXsSmem);
  if (e != cudaSuccess) return launch_error(e);
  if (per_sm < 1) return SO101_ERR_LAUNCH;

  XsParams p;
  memset(&p, 0, sizeof(p));
  for (int l = 0; l < s->n_layers; ++l) {
    const so101_expert_layer& y = s->layer[l];
    const long long rows_in = s->q_dim + (y.self_attn ? 2LL * s->kv_dim : 0);
    if ((rc = xs_map(&p.maps[l][kXsAttnIn], y.w_attn, rows_in, s->exp_dim)) ||
        (rc = xs_map(&p.maps[l][kXsO], y.w_o, s->exp_dim, s->q_dim)) ||
        (rc = xs_map(&p.maps[l][kXsGateUp], y.w_gate_up, 2LL * s->mlp_dim, s->exp_dim)) ||
        (rc = xs_map(&p.maps[l][kXsDown], y.w_down, s->exp_dim, s->mlp_dim)))
      return rc;
    p.layer[l].ln_in = y.ln_in;
    p.layer[l].ln_post = y.ln_post;
    p.layer[l].k = static_cast<__nv_bfloat16*>(y.k);
    p.layer[l].v = static_cast<__nv_bfloat16*>(y.v);
    p.layer[l].self_attn = y.self_attn != 0;
  }
  if ((rc = xs_map(&p.tm_attn, s->attn, s->rows, s->q_dim, 64)) || (rc = xs_map(&p.tm_act, s->act, s->rows, s->mlp_dim, 64)))
    return rc;
  uint8_t* ws = static_cast<uint8_t*>(s->workspace);
  p.e = s->e;
  p.q = static_cast<__nv_bfloat16*>(s->q);
  p.attn = static_cast<__nv_bfloat16*>(s->attn);
  p.act = static_cast<__nv_bfloat16*>(s->act);
  p.partials = reinterpret_cast<float*>(ws + lay.partials);
  p.tickets = reinterpret_cast<int*>(ws + lay.tickets);
  p.bar = reinterpret_cast<unsigned*>(ws + lay.bar);
  p.ss = reinterpret_cast<float*>(ws + lay.ss);
  p.cos_s = s->cos_self;
  p.sin_s = s->sin_self;
  p.cos_c = s->cos_cross;
  p.sin_c = s->sin_cross;
  p.n_layers = s->n_layers;
  p.H = s->rows;
  p.L = s->prefix_len;
  p.D = s->exp_dim;
  p.QD = s->q_dim;
  p.KV = s->kv_dim;
  p.F = s->mlp_dim;
  p.nq = s->n_heads;
  p.nkv = s->n_kv;
  p.kbs[kXsAttnIn] = xs_kbs(s->q_dim + 2 * s->kv_dim, s->exp_dim, sms);
  p.kbs[kXsO] = xs_kbs(s->exp_dim, s->q_dim, sms);
  p.kbs[kXsGateUp] = xs_kbs(s->mlp_dim, s->exp_dim, sms);
  p.kbs[kXsDown] = xs_kbs(s->exp_dim, s->mlp_dim, sms);
  p.eps = s->eps;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / 8.0);
  p.status = status_ptr();
  p.wait_ns = g_xs_wait_ns > 0 ? static_cast<unsigned long long>(g_xs_wait_ns) : kWaitLimitNs;
  p.withhold = g_xs_withhold < sms ? g_xs_withhold : -1;
  // tickets and barrier state start at zero (a launch that aborted may have left them set)
  e = cudaMemsetAsync(ws + lay.tickets, 0, static_cast<size_t>(lay.ss - lay.tickets), stream);
  if (e != cudaSuccess) return launch_error(e);

  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(sms), 1, 1);
  lc.blockDim = dim3(kXsThreads, 1, 1);
  lc.dynamicSmemBytes = kXsSmem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid barriers need it
  attr[0].val.cooperative = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  e = cudaLaunchKernelEx(&lc, expert_step_kernel, p);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}

extern "C" int so101_expert_step_test_hooks(int64_t wait_limit_ns, int withhold_cta) {
  if (wait_limit_ns < 0 || wait_limit_ns > static_cast<int64_t>(kWaitLimitNs) || withhold_cta < -1)
    return SO101_ERR_ARG;
  g_xs_wait_ns = wait_limit_ns;
  g_xs_withhold = withhold_cta;
  return SO101_OK;
}
