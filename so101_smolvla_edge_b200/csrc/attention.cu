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

template <int HD, bool SPLIT>
__global__ void __launch_bounds__(128) attention_kernel(const AttnArgs a) {
  constexpr int BM = 64, BN = 64, LDS = HD + 8, HALF = HD / 2;
  constexpr int CHUNKS = HD / 8;  // 16-byte chunks per row
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw);
  __nv_bfloat16* sK = sQ + BM * LDS;          // [2][BN * LDS]
  __nv_bfloat16* sV = sK + 2 * BN * LDS;      // [2][BN * LDS]

  grid_dep_launch();
  grid_dep_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = SPLIT ? a.kv_splits : 1;
  const int split = S > 1 ? static_cast<int>(blockIdx.x % S) : 0;
  const int q0 = (S > 1 ? blockIdx.x / S : blockIdx.x) * BM, h = blockIdx.y, bi = blockIdx.z;
  const int kvh = h / (a.nq / a.nkv);
  const __nv_bfloat16* Q = a.q + bi * a.bq + static_cast<long long>(h) * HD;
  const __nv_bfloat16* K = a.k + bi * a.bk + static_cast<long long>(kvh) * HD;
  const __nv_bfloat16* V = a.v + bi * a.bv + static_cast<long long>(kvh) * HD;

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
    for (int c = tid; c < BN * CHUNKS; c += 128) {
      const int r = c / CHUNKS, cc = c % CHUNKS;
      const int j = j0 + r;
      const bool ok = j < a.Lk;
      const long long jj = ok ? j : 0;
      cp_async16(smem_u32(sK + buf * BN * LDS + r * LDS + cc * 8), K + jj * a.ldk + cc * 8, ok ? 16 : 0);
      cp_async16(smem_u32(sV + buf * BN * LDS + r * LDS + cc * 8), V + jj * a.ldv + cc * 8, ok ? 16 : 0);
    }
    cp_async_commit();
  };

  if (n_tiles > 0) load_kv(t_begin, 0);

  // stage Q (rotated) into shared memory: 8 dims of each rotary half per step, 16-byte loads
  constexpr int VH = HALF / 8;
  for (int idx = tid; idx < BM * VH; idx += 128) {
    const int r = idx / VH, d0 = (idx % VH) * 8;
    const int i = q0 + r;
    uint4 o1 = make_uint4(0, 0, 0, 0), o2 = o1;
    if (i < a.Lq) {
      const __nv_bfloat16* qr = Q + static_cast<long long>(i) * a.ldq;
      const uint4 u1 = *reinterpret_cast<const uint4*>(qr + d0);
      const uint4 u2 = *reinterpret_cast<const uint4*>(qr + d0 + HALF);
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

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < n_tiles) {
      load_kv(t_begin + tile + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
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
    // scale, mask, row max
    const int j0 = (t_begin + tile) * BN;
    float mx0 = -INFINITY, mx1 = -INFINITY;
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
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - base0), al1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int t = 0; t < BN / 8; ++t) {
      const float p0 = exp2f(s[t][0] - base0), p1 = exp2f(s[t][1] - base0);
      const float p2 = exp2f(s[t][2] - base1), p3 = exp2f(s[t][3] - base1);
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
    __syncthreads();  // this buffer is refilled two tiles from now
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
    float* sW = sML + 2 * BM;                    // [64][8]: merge weights
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
    // CTA `split` merges rows [split*64/S, (split+1)*64/S) over all splits, in split order
    const int rlo = split * BM / S, rhi = (split + 1) * BM / S, nr = rhi - rlo;
    const uint32_t o_addr = smem_u32(sO), ml_addr = smem_u32(sML);
    if (tid < nr) {
      const int r = rlo + tid;
      float ms[8], ls[8], mx = -INFINITY;
#pragma unroll
      for (int sp = 0; sp < 8; ++sp) {
        if (sp < S) {
          const uint32_t pa = mapa_shared(ml_addr, static_cast<uint32_t>(sp)) + static_cast<uint32_t>(8 * r);
          ms[sp] = ld_cluster_f32(pa);
          ls[sp] = ld_cluster_f32(pa + 4);
          mx = fmaxf(mx, ms[sp]);
        }
      }
      if (mx == -INFINITY) mx = 0.f;
      float l = 0.f;
#pragma unroll
      for (int sp = 0; sp < 8; ++sp) {
        if (sp < S) {
          ms[sp] = exp2f(ms[sp] - mx);
          l += ls[sp] * ms[sp];
        }
      }
      const float inv = 1.f / l;
#pragma unroll
      for (int sp = 0; sp < 8; ++sp) sW[8 * tid + sp] = sp < S ? ms[sp] * inv : 0.f;
    }
    __syncthreads();
    for (int idx = tid; idx < nr * (HD / 4); idx += 128) {
      const int rr = idx / (HD / 4), c4 = (idx % (HD / 4)) * 4;
      const int row = q0 + rlo + rr;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float4 part[8];
#pragma unroll
      for (int sp = 0; sp < 8; ++sp)
        if (sp < S)
          part[sp] = ld_cluster_f32x4(mapa_shared(o_addr, static_cast<uint32_t>(sp)) +
                                      static_cast<uint32_t>(((rlo + rr) * LDO + c4) * 4));
#pragma unroll
      for (int sp = 0; sp < 8; ++sp) {
        if (sp < S) {
          const float wgt = sW[8 * rr + sp];
          acc.x += part[sp].x * wgt, acc.y += part[sp].y * wgt, acc.z += part[sp].z * wgt, acc.w += part[sp].w * wgt;
        }
      }
      if (row < a.Lq) {
        const long long off = obase + static_cast<long long>(row) * a.ldo + c4;
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
    cluster_sync();  // peers keep their shared memory until every merge has read it
    return;
  }
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
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

template <int HD>
int launch_attention(const AttnArgs& a, int batch, cudaStream_t stream) {
  constexpr int smem = (64 * (HD + 8) + 4 * 64 * (HD + 8)) * 2;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_kernel<HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  const int q_tiles = (a.Lq + 63) / 64;
  dim3 grid(q_tiles * a.kv_splits, a.nq, batch);
  if (a.kv_splits == 1) return launch_kernel(attention_kernel<HD, false>, dim3(grid), dim3(128), smem, stream, a);
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = dim3(128);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.kv_splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&lc, attention_kernel<HD, true>, a);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}

bool attention_tc_eligible(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                           long long Lq, long long Lk, int nq, int nkv, int hd, long long causal_from,
                           const float* cos, long long bq, long long bk, long long bv, int o_type);
int attention_tc_launch(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                        void* o, long long ldo, int o_type, float o_qscale, long long L, int heads, int batch,
                        cudaStream_t stream);

}  // namespace so101

using namespace so101;

extern "C" int so101_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                               void* o, int64_t ldo, int o_type, float o_qscale, int64_t Lq, int64_t Lk, int nq,
                               int nkv, int hd, int64_t causal_from, int64_t q_offset, const float* cos,
                               const float* sin, int batch, int64_t bq, int64_t bk, int64_t bv, int64_t bo,
                               cudaStream_t stream) {
  if (!q || !k || !v || !o || Lq <= 0 || Lk <= 0 || nq <= 0 || nkv <= 0 || nq % nkv || batch <= 0) return SO101_ERR_ARG;
  if (hd != 32 && hd != 64 && hd != 128) return SO101_ERR_ARG;
  if ((cos == nullptr) != (sin == nullptr)) return SO101_ERR_ARG;
  if (o_type != SO101_BF16 && o_type != SO101_I8) return SO101_ERR_ARG;
  if (o_type == SO101_I8 && !(o_qscale > 0.f)) return SO101_ERR_ARG;
  if (Lq > (1 << 30) || Lk > (1 << 30) || nq > 65535 || batch > 65535) return SO101_ERR_ARG;
  // 16-byte cp.async rows: K/V bases (with the head offset) and row strides
  if (reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16 || (ldk * 2) % 16 ||
      (ldv * 2) % 16 || (bk * 2) % 16 || (bv * 2) % 16)
    return SO101_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(o) % 4 || ldo % 2 || bo % 2) return SO101_ERR_ARG;
  // q rows and the rotary tables are read in 16-byte pieces
  if (reinterpret_cast<uintptr_t>(q) % 16 || (ldq * 2) % 16 || (bq * 2) % 16) return SO101_ERR_ARG;
  if (cos && (reinterpret_cast<uintptr_t>(cos) % 16 || reinterpret_cast<uintptr_t>(sin) % 16)) return SO101_ERR_ARG;
  if (attention_tc_eligible(q, ldq, k, ldk, v, ldv, Lq, Lk, nq, nkv, hd, causal_from, cos, bq, bk, bv, o_type) &&
      ldo % 8 == 0 && bo == Lq * ldo && reinterpret_cast<uintptr_t>(o) % 16 == 0)
    return attention_tc_launch(q, ldq, k, ldk, v, ldv, o, ldo, o_type, o_qscale, Lq, nq, batch, stream);
  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.o = o;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.ldo = ldo;
  a.bq = bq;
  a.bk = bk;
  a.bv = bv;
  a.bo = bo;
  a.o_type = o_type;
  a.o_qscale = o_qscale;
  a.Lq = static_cast<int>(Lq);
  a.Lk = static_cast<int>(Lk);
  a.nq = nq;
  a.nkv = nkv;
  a.causal_from = causal_from;
  a.q_offset = q_offset;
  a.cos = cos;
  a.sin = sin;
  a.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(hd)));
  // few CTAs (the expert's 50 queries, the 241-row prefix): split the key tiles over a cluster
  {
    long long last = causal_from - 1;
    if (Lq - 1 + q_offset > last) last = Lq - 1 + q_offset;
    if (last > Lk - 1) last = Lk - 1;
    const long long tiles = (last + 64) / 64;
    const long long ctas = ((Lq + 63) / 64) * static_cast<long long>(nq) * batch;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long sp = ctas >= sms ? 1 : (sms + ctas - 1) / ctas;
    if (sp > tiles) sp = tiles;
    if (sp > 8) sp = 8;
    if (sp < 1) sp = 1;
    const long long per = (tiles + sp - 1) / sp;
    a.kv_splits = static_cast<int>((tiles + per - 1) / per);  // no split without key tiles
  }
  switch (hd) {
    case 32: return launch_attention<32>(a, batch, stream);
    case 64: return launch_attention<64>(a, batch, stream);
    default: return launch_attention<128>(a, batch, stream);
  }
}
