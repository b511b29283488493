// Cluster reduction of per-CTA fp32 partials of one 128-feature output tile, by whole tokens, with
// the residual epilogue of the fused expert kernels (attention_o.cu, mlp.cu).
//
// Every CTA of the cluster holds its partial in its own shared memory, column-major with a token's
// 128 features contiguous (part[token * 128 + feature]). CTA r of S owns tokens
// [r*nv/S, (r+1)*nv/S); warp w takes one token at a time, lane l features 4l..4l+3. Per token the
// S partials are summed in cluster-rank order (deterministic), then
//   y[row, n]   = sum + residual[row, n]                (fp32)
//   y16[row, n] = bf16(y[row, n] * y16_scale[n])        (the next RMSNorm's weight; optional)
//   stat_ss[row * stat_ld + tile] = sum over the tile's features of y^2   (optional)
// with row = row0 + token: one statistics slot per output tile. n_out must be a multiple of 4 and
// the row pieces 16-byte (y, residual) / 8-byte (y16) aligned; the caller checks both.
#pragma once

#include "common.cuh"

namespace so101 {

struct TokenEpilogue {
  float* y;
  long long ldy;
  const float* res;
  long long ldr;
  __nv_bfloat16* y16;
  long long ld16;
  const float* y16_scale;
  float* stat_ss;
  long long stat_ld;
  int n_out;
};

// A thread's residual pieces for its warp's first two tokens and its y16 scales, loaded early (any
// time after the residual's producer is complete) so the reduction waits on DSMEM alone.
struct TokenPrefetch {
  float4 res[2];
  float4 scale;
};

template <int THREADS>
__device__ __forceinline__ TokenPrefetch token_prefetch(const TokenEpilogue& e, int S, int nv, long long row0, int tile) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int lo = rank * nv / S, hi = (rank + 1) * nv / S;
  const int n = tile * 128 + lane * 4;
  const bool n_ok = n < e.n_out;
  TokenPrefetch pf;
#pragma unroll
  for (int it = 0; it < 2; ++it) {
    const int tok = lo + warp + it * (THREADS / 32);
    pf.res[it] = (n_ok && e.res && tok < hi)
                     ? *reinterpret_cast<const float4*>(e.res + (row0 + tok) * e.ldr + n)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pf.scale = (n_ok && e.y16_scale) ? __ldg(reinterpret_cast<const float4*>(e.y16_scale + n))
                                   : make_float4(1.f, 1.f, 1.f, 1.f);
  return pf;
}

// All threads of every CTA call it between two cluster barriers (the first publishes the partials,
// the second keeps them alive until every peer has read them); pf from token_prefetch with the same
// arguments.
template <int MAXS, int THREADS>
__device__ __forceinline__ void cluster_token_reduce(const TokenEpilogue& e, const float* part, int S, int nv,
                                                     long long row0, int tile, const TokenPrefetch& pf) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int lo = rank * nv / S, hi = (rank + 1) * nv / S;
  const uint32_t part_addr = smem_u32(part);
  uint32_t peer[MAXS];
#pragma unroll
  for (int sp = 0; sp < MAXS; ++sp) peer[sp] = mapa_shared(part_addr, static_cast<uint32_t>(sp < S ? sp : 0));
  const int n = tile * 128 + lane * 4;
  const bool n_ok = n < e.n_out;
#pragma unroll 1
  for (int tok = lo + warp, it = 0; tok < hi; tok += THREADS / 32, ++it) {
    const uint32_t off = static_cast<uint32_t>((tok * 128 + lane * 4) * 4);
    const long long row = row0 + tok;
    float4 pv[MAXS];
    float4 r = it == 0 ? pf.res[0] : pf.res[1];
    if (n_ok) {
#pragma unroll
      for (int sp = 0; sp < MAXS; ++sp)
        if (sp < S) pv[sp] = ld_cluster_f32x4(peer[sp] + off);
      if (e.res && it >= 2) r = *reinterpret_cast<const float4*>(e.res + row * e.ldr + n);
    }
    float ss = 0.f;
    if (n_ok) {
      float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sp = 0; sp < MAXS; ++sp)
        if (sp < S) s.x += pv[sp].x, s.y += pv[sp].y, s.z += pv[sp].z, s.w += pv[sp].w;
      const float4 x = make_float4(s.x + r.x, s.y + r.y, s.z + r.z, s.w + r.w);
      *reinterpret_cast<float4*>(e.y + row * e.ldy + n) = x;
      if (e.y16) {
        const float4 c = pf.scale;
        __nv_bfloat162 hv[2] = {__floats2bfloat162_rn(x.x * c.x, x.y * c.y), __floats2bfloat162_rn(x.z * c.z, x.w * c.w)};
        *reinterpret_cast<uint2*>(e.y16 + row * e.ld16 + n) = *reinterpret_cast<uint2*>(hv);
      }
      ss = (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0 && e.stat_ss) e.stat_ss[row * e.stat_ld + tile] = ss;
  }
}

}  // namespace so101
