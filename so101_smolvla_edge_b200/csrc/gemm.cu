// tcgen05 GEMM for sm_100a: y = epilogue(x @ w^T), TMA-fed shared-memory ring, TMEM accumulator.
//
// Two kernels serve every linear of the chunk.
//
// gemm_tc_kernel (one output tile per CTA, 128 threads)
//   normal  (SWAP = false)  token rows on the 128-row MMA M side, features on MMA N (BN).
//   swap    (SWAP = true)   weight rows on the 128-row MMA M side, the few token rows (<= 64, the
//                           action expert's 50) on MMA N: weight streaming, each CTA reads a
//                           128 x K slab of W once and the 50 rows never pad to 128.
//   split-K over grid.z, deterministic, two ways:
//     cluster  the splits of a tile form one thread-block cluster; each CTA stages its fp32
//              partial in its own shared memory, and after a cluster barrier CTA r sums rows
//              [r*128/S, (r+1)*128/S) over all S CTAs in split order (DSMEM reads) and runs the
//              epilogue for them. No global round trip, no workspace.
//     global   each split stores its partial to a workspace and takes a ticket; the last split to
//              arrive sums all partials in split order, runs the epilogue and zeroes the ticket.
//   Warp roles: warp 0 lane 0 issues TMA, warp 1 lane 0 issues tcgen05.mma and owns TMEM; all four
//   warps run the epilogue, warp w reading TMEM lanes [32w, 32w+32).
//
// gemm_persistent_kernel (normal tiling for large M, 1 CTA per SM, 320 threads)
//   Each CTA loops over output tiles. Warp 0 streams A/B tiles through the ring, warp 1 issues the
//   MMAs into one of two TMEM accumulators (2 x BN columns) and sixteen epilogue warps drain the
//   other, so the epilogue of tile i overlaps the MMAs of tile i+1. Epilogue warp e reads lane
//   quadrant (e + 2) % 4 and column quarter e / 4 into registers in one go and releases the
//   accumulator before its arithmetic.
//
// DUAL (SiLU gate): two weight tiles per stage (gate rows n and up rows N + n of the fused
// [gate; up] matrix) into two accumulators; the epilogue writes silu(gate) * up.
// Shared-memory tiles are 128-byte K rows in TMA SWIZZLE_128B layout, the canonical K-major layout
// the MMA descriptors name. No TMA multicast anywhere.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace so101 {

constexpr int kMaxSplitCluster = 8;  // portable cluster size: the most K splits reduced on chip

struct GemmArgs {
  int M, N, K;  // N: output features (half of w's rows for SILU_GATE)
  int kb_total, kb_per_split, splits, tiles_q, num_tiles;
  void* y;
  long long ldy;
  int y_type;
  int epilogue;
  const float* bias;
  const void* res;
  long long ldr;
  int r_type;
  long long r_period;
  float out_scale;
  const float* w_scale;
  float x_scale;
  float y_qscale, y_qinv;
  long long row_group, row_stride;
  void* ws;
  int* tickets;
  int vec_ok;
  int cluster_reduce;
  int* status;
  // RMSNorm folded into the GEMM: v *= rsqrt(sum of rms_slots sums of squares / rms_n + rms_eps)
  const float* rms_ss;
  int rms_slots;
  long long rms_ld;
  float rms_n, rms_eps;
  // producer side: per-slot sums of squares of the final rows, and a bf16 copy of the output
  float* stat_ss;
  long long stat_ld;
  void* y16;
  long long ld16;
  const float* y16_scale;  // per output column (the next norm's weight), NULL: 1
};

// Per-token RMSNorm scale from the producer's sums of squares: token m's slots are contiguous
// (row m of rms_ss, stride rms_ld, a multiple of 4, at most 64 slots); all of them are loaded at once
// and summed in slot order.
__device__ __forceinline__ float rms_scale(const GemmArgs& a, long long m) {
  const float4* row = reinterpret_cast<const float4*>(a.rms_ss + m * a.rms_ld);
  float4 v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = 4 * i < a.rms_slots ? row[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float x[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (4 * i + j < a.rms_slots) s += x[j];
  }
  return rsqrtf(s / a.rms_n + a.rms_eps);
}

__device__ __forceinline__ float load_elem(const void* p, long long i, int type) {
  if (type == SO101_F32) return static_cast<const float*>(p)[i];
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ long long out_row(const GemmArgs& a, int m) {
  return a.row_group > 0 ? (m / a.row_group) * a.row_stride + m % a.row_group : m;
}

// Epilogue of one accumulator element (m, n); u is the up-projection accumulator for SILU_GATE.
template <bool DUAL, bool I8>
__device__ __forceinline__ void epilogue1(const GemmArgs& a, int m, int n, float v, float u, float rs = 1.f) {
  if (m >= a.M || n >= a.N) return;
  v *= rs;
  u *= rs;
  float x = v;
  if (I8) x *= a.x_scale * __ldg(a.w_scale + n);
  if (a.bias) x += __ldg(a.bias + n);
  if (a.epilogue == SO101_EPI_GELU) {
    x = gelu_tanh(x);
  } else if (DUAL) {
    float up = u;
    if (I8) up *= a.x_scale * __ldg(a.w_scale + a.N + n);
    x = silu(x) * up;
  }
  x *= a.out_scale;
  const long long row = out_row(a, m);
  if (a.res) {
    const long long rrow = a.r_period > 0 ? m % a.r_period : row;
    x += load_elem(a.res, rrow * a.ldr + n, a.r_type);
  }
  const long long i = row * a.ldy + n;
  if (a.y_type == SO101_F32)
    static_cast<float*>(a.y)[i] = x;
  else if (a.y_type == SO101_BF16)
    static_cast<__nv_bfloat16*>(a.y)[i] = __float2bfloat16_rn(x);
  else
    static_cast<int8_t*>(a.y)[i] = static_cast<int8_t>(quant_i8_int(x, a.y_qscale, a.y_qinv));
}

// Epilogue of 16 accumulator values sharing P index p, Q indices [qb, qb + 16).
template <bool SWAP, bool DUAL, bool I8>
__device__ __forceinline__ void epilogue16(const GemmArgs& a, int p, int qb, float (&v)[16], float (&u)[16],
                                          const float* rtab = nullptr, int rbase = 0) {
  if (rtab) {  // RMSNorm scale of each element's token (q for SWAP, p otherwise)
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float rs = rtab[(SWAP ? qb + j : p) - rbase];
      v[j] *= rs;
      u[j] *= rs;
    }
  }
  if (!SWAP) {
    const int m = p;
    if (m >= a.M) return;
    if (a.vec_ok && qb + 16 <= a.N) {
      const long long row = out_row(a, m);
      const long long rrow = a.r_period > 0 ? m % a.r_period : row;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = qb + j;
        float x = v[j];
        if (I8) x *= a.x_scale * __ldg(a.w_scale + n);
        if (a.bias) x += __ldg(a.bias + n);
        if (a.epilogue == SO101_EPI_GELU) {
          x = gelu_tanh(x);
        } else if (DUAL) {
          float up = u[j];
          if (I8) up *= a.x_scale * __ldg(a.w_scale + a.N + n);
          x = silu(x) * up;
        }
        v[j] = x * a.out_scale;
      }
      if (a.res) {
        if (a.r_type == SO101_F32) {
          const float4* r4 = reinterpret_cast<const float4*>(static_cast<const float*>(a.res) + rrow * a.ldr + qb);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 r = r4[j];
            v[4 * j] += r.x;
            v[4 * j + 1] += r.y;
            v[4 * j + 2] += r.z;
            v[4 * j + 3] += r.w;
          }
        } else {
          const uint4* r4 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.res) + rrow * a.ldr + qb);
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            uint4 r = r4[j];
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __bfloat1622float2(h[e]);
              v[8 * j + 2 * e] += f.x;
              v[8 * j + 2 * e + 1] += f.y;
            }
          }
        }
      }
      if (a.y_type == SO101_F32) {
        float4* y4 = reinterpret_cast<float4*>(static_cast<float*>(a.y) + row * a.ldy + qb);
#pragma unroll
        for (int j = 0; j < 4; ++j) y4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else if (a.y_type == SO101_BF16) {
        uint4 o[2];
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        uint4* y4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.y) + row * a.ldy + qb);
        y4[0] = o[0];
        y4[1] = o[1];
      } else {
        uint32_t w4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t b0 = quant_i8_int(v[4 * e], a.y_qscale, a.y_qinv) & 0xFF;
          const uint32_t b1 = quant_i8_int(v[4 * e + 1], a.y_qscale, a.y_qinv) & 0xFF;
          const uint32_t b2 = quant_i8_int(v[4 * e + 2], a.y_qscale, a.y_qinv) & 0xFF;
          const uint32_t b3 = quant_i8_int(v[4 * e + 3], a.y_qscale, a.y_qinv) & 0xFF;
          w4[e] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
        *reinterpret_cast<uint4*>(static_cast<int8_t*>(a.y) + row * a.ldy + qb) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
      }
      return;
    }
  }
#pragma unroll 4
  for (int j = 0; j < 16; ++j) {
    const int q = qb + j;
    epilogue1<DUAL, I8>(a, SWAP ? q : p, SWAP ? p : q, v[j], u[j]);
  }
}

// Lean epilogue of 16 consecutive output columns of row m (tokens on the MMA M side), for chunks
// fully inside N with vector-aligned rows. kc / kb / ku hold this chunk's per-column constants in
// shared memory: the dequantization scale (x_scale * w_scale[n], int8 only), the bias, and the
// up-projection scale (int8 SiLU gate).
// Values of 16 consecutive output columns of one row before the residual: dequantization scale,
// bias, RMSNorm row scale, SiLU gate or GELU, out_scale. Shared by the row-per-lane stores below and
// the transposed stores of the CTA-pair kernel, so both round identically.
template <bool DUAL, bool I8>
__device__ __forceinline__ void epilogue_values16(const GemmArgs& a, const uint32_t (&r0)[16], const uint32_t (&r1)[16],
                                                  const float* kc, const float* kb, const float* ku, float rs,
                                                  float (&v)[16]) {
  // packed fp32x2 throughout (the epilogue is instruction-bound); rs differs from 1 only with a
  // folded RMSNorm, and multiplying by 1 is exact, so that multiply is skipped without it
  const bool scaled = a.rms_ss != nullptr;
  const float2 rs2 = make_float2(rs, rs);
  float2 x[8];
#pragma unroll
  for (int j4 = 0; j4 < 4; ++j4) {
    const float4 bi = *reinterpret_cast<const float4*>(kb + 4 * j4);
    float2 s01, s23, x01, x23;
    if constexpr (I8) {
      const float4 sc = *reinterpret_cast<const float4*>(kc + 4 * j4);
      s01 = make_float2(sc.x, sc.y);
      s23 = make_float2(sc.z, sc.w);
      if (scaled) {
        s01 = fmul2(s01, rs2);
        s23 = fmul2(s23, rs2);
      }
      x01 = make_float2(static_cast<float>(static_cast<int>(r0[4 * j4])), static_cast<float>(static_cast<int>(r0[4 * j4 + 1])));
      x23 = make_float2(static_cast<float>(static_cast<int>(r0[4 * j4 + 2])), static_cast<float>(static_cast<int>(r0[4 * j4 + 3])));
    } else {
      s01 = s23 = rs2;
      x01 = make_float2(__uint_as_float(r0[4 * j4]), __uint_as_float(r0[4 * j4 + 1]));
      x23 = make_float2(__uint_as_float(r0[4 * j4 + 2]), __uint_as_float(r0[4 * j4 + 3]));
    }
    x[2 * j4] = ffma2(x01, s01, make_float2(bi.x, bi.y));
    x[2 * j4 + 1] = ffma2(x23, s23, make_float2(bi.z, bi.w));
  }
  if constexpr (DUAL) {
    // the SiLU gate stays scalar: packed it measured slower (the pair packing costs moves here)
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      float su[4] = {rs, rs, rs, rs};
      if constexpr (I8) {
        const float4 sc = *reinterpret_cast<const float4*>(ku + 4 * j4);
        su[0] = sc.x * rs, su[1] = sc.y * rs, su[2] = sc.z * rs, su[3] = sc.w * rs;
      }
      float g[4] = {x[2 * j4].x, x[2 * j4].y, x[2 * j4 + 1].x, x[2 * j4 + 1].y};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float up = I8 ? static_cast<float>(static_cast<int>(r1[4 * j4 + e])) * su[e]
                            : __uint_as_float(r1[4 * j4 + e]) * su[e];
        g[e] = silu(g[e]) * up;
      }
      x[2 * j4] = make_float2(g[0], g[1]);
      x[2 * j4 + 1] = make_float2(g[2], g[3]);
    }
  } else if (a.epilogue == SO101_EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = gelu_tanh_fast2(x[j]);
  }
  if (a.out_scale != 1.f) {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = fmul2(x[j], make_float2(a.out_scale, a.out_scale));
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) v[2 * j] = x[j].x, v[2 * j + 1] = x[j].y;
}

template <bool DUAL, bool I8>
__device__ __forceinline__ float epilogue_row16_fast(const GemmArgs& a, int m, int qb, const uint32_t (&r0)[16],
                                                     const uint32_t (&r1)[16], const float* kc, const float* kb,
                                                     const float* ku, float rs = 1.f) {
  float v[16];
  epilogue_values16<DUAL, I8>(a, r0, r1, kc, kb, ku, rs, v);
  const long long row = out_row(a, m);
  if (a.res) {
    const long long rrow = a.r_period > 0 ? m % a.r_period : row;
    if (a.r_type == SO101_F32) {
      const float4* r4 = reinterpret_cast<const float4*>(static_cast<const float*>(a.res) + rrow * a.ldr + qb);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 r = r4[j];
        const float2 s01 = fadd2(make_float2(v[4 * j], v[4 * j + 1]), make_float2(r.x, r.y));
        const float2 s23 = fadd2(make_float2(v[4 * j + 2], v[4 * j + 3]), make_float2(r.z, r.w));
        v[4 * j] = s01.x, v[4 * j + 1] = s01.y, v[4 * j + 2] = s23.x, v[4 * j + 3] = s23.y;
      }
    } else {
      const uint4* r4 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.res) + rrow * a.ldr + qb);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        uint4 r = r4[j];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          v[8 * j + 2 * e] += f.x, v[8 * j + 2 * e + 1] += f.y;
        }
      }
    }
  }
  if (a.y_type == SO101_F32) {
    float4* y4 = reinterpret_cast<float4*>(static_cast<float*>(a.y) + row * a.ldy + qb);
#pragma unroll
    for (int j = 0; j < 4; ++j) y4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  } else if (a.y_type == SO101_BF16) {
    uint4 o[2];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    uint4* y4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.y) + row * a.ldy + qb);
    y4[0] = o[0];
    y4[1] = o[1];
  } else {
    const float inv = a.y_qinv;
    *reinterpret_cast<uint4*>(static_cast<int8_t*>(a.y) + row * a.ldy + qb) =
        make_uint4(pack4_i8(v[0], v[1], v[2], v[3], inv), pack4_i8(v[4], v[5], v[6], v[7], inv),
                   pack4_i8(v[8], v[9], v[10], v[11], inv), pack4_i8(v[12], v[13], v[14], v[15], inv));
  }
  float ssq = 0.f;
  if (a.stat_ss) {
#pragma unroll
    for (int j = 0; j < 16; ++j) ssq = fmaf(v[j], v[j], ssq);
  }
  if (a.y16) {
    float c[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) c[j] = 1.f;
    if (a.y16_scale) {
      const float4* s4 = reinterpret_cast<const float4*>(a.y16_scale + qb);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 s = __ldg(s4 + j);
        c[4 * j] = s.x, c[4 * j + 1] = s.y, c[4 * j + 2] = s.z, c[4 * j + 3] = s.w;
      }
    }
    uint4 o[2];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = __floats2bfloat162_rn(v[2 * e] * c[2 * e], v[2 * e + 1] * c[2 * e + 1]);
    uint4* y4 = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.y16) + row * a.ld16 + qb);
    y4[0] = o[0];
    y4[1] = o[1];
  }
  return ssq;
}

// Residual, output, bf16 copy and sum of squares of 4 consecutive columns [n, n + 4) of row m
// (vector path: n + 4 <= N, aligned rows), from values as epilogue_values16 leaves them.
__device__ __forceinline__ float epilogue_store4(const GemmArgs& a, int m, int n, float4 x) {
  const long long row = out_row(a, m);
  if (a.res) {
    const long long rrow = a.r_period > 0 ? m % a.r_period : row;
    if (a.r_type == SO101_F32) {
      const float4 r = *reinterpret_cast<const float4*>(static_cast<const float*>(a.res) + rrow * a.ldr + n);
      const float2 s01 = fadd2(make_float2(x.x, x.y), make_float2(r.x, r.y));
      const float2 s23 = fadd2(make_float2(x.z, x.w), make_float2(r.z, r.w));
      x = make_float4(s01.x, s01.y, s23.x, s23.y);
    } else {
      const uint2 r = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(a.res) + rrow * a.ldr + n);
      const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
      x.x += f0.x, x.y += f0.y, x.z += f1.x, x.w += f1.y;
    }
  }
  if (a.y_type == SO101_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(a.y) + row * a.ldy + n) = x;
  } else if (a.y_type == SO101_BF16) {
    __nv_bfloat162 h[2] = {__floats2bfloat162_rn(x.x, x.y), __floats2bfloat162_rn(x.z, x.w)};
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.y) + row * a.ldy + n) = *reinterpret_cast<uint2*>(h);
  } else {
    *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(a.y) + row * a.ldy + n) = pack4_i8(x.x, x.y, x.z, x.w, a.y_qinv);
  }
  if (a.y16) {
    const float4 c = a.y16_scale ? __ldg(reinterpret_cast<const float4*>(a.y16_scale + n)) : make_float4(1.f, 1.f, 1.f, 1.f);
    __nv_bfloat162 h[2] = {__floats2bfloat162_rn(x.x * c.x, x.y * c.y), __floats2bfloat162_rn(x.z * c.z, x.w * c.w)};
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.y16) + row * a.ld16 + n) = *reinterpret_cast<uint2*>(h);
  }
  return (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
}

template <bool I8>
__device__ __forceinline__ float acc_value(uint32_t r) {
  return I8 ? i32_to_f32(static_cast<int>(r)) : __uint_as_float(r);
}

// ================================================================ one tile per CTA
// 256 threads: warp 0 issues TMA, warp 1 the MMAs; in the epilogue every TMEM lane (row of the
// 128-row tile) has two threads, one per half of the columns (warps 4-7 read the same lane
// quadrants as warps 0-3), and the cluster reduction covers twice the items per DSMEM round trip.
// Two CTAs fit per SM (at most 128 registers) except with the SiLU gate on swap tiles, whose two
// accumulators' split partials need more registers and whose grids are small (M <= 64).
constexpr int kTileThreads = 256;

template <int BN, bool SWAP, bool DUAL, bool I8>
__global__ void __launch_bounds__(kTileThreads, (SWAP && DUAL) ? 1 : 2)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                   const GemmArgs a, const int stages) {
  constexpr int NA = (SWAP && DUAL) ? 2 : 1;   // tiles on the MMA M side per stage
  constexpr int NB = (!SWAP && DUAL) ? 2 : 1;  // tiles on the MMA N side per stage
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = BN * 128;
  constexpr int STAGE_BYTES = NA * A_BYTES + NB * B_BYTES;
  constexpr int NACC = BN * (DUAL ? 2 : 1);
  constexpr uint32_t TMEM_COLS = NACC <= 32 ? 32 : NACC <= 64 ? 64 : NACC <= 128 ? 128 : NACC <= 256 ? 256 : 512;
  constexpr uint32_t IDESC = I8 ? idesc_i8(128, BN) : idesc_bf16(128, BN);
  constexpr int KB_ELEMS = I8 ? 128 : 64;  // 128 bytes of K per stage

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * STAGE_BYTES);
  uint64_t* empty = full + stages;
  uint64_t* accum = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  // epilogue scratch past the barriers: the RMSNorm scale of this tile's tokens, and the
  // statistics reduction of the cluster path
  float* rtab_s = reinterpret_cast<float*>(smem + stages * STAGE_BYTES + 256);
  float* stat_red = rtab_s + 128;  // [BN][32]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q_tile = blockIdx.x, p_tile = blockIdx.y, split = blockIdx.z;
  const int p0 = p_tile * 128, q0 = q_tile * BN;
  const int rbase = SWAP ? q0 : p0;
  const int kb0 = split * a.kb_per_split;
  const int kb1 = min(kb0 + a.kb_per_split, a.kb_total);
  const int nkb = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_launch();  // the next kernel may start its own prologue and weight prefetch

  if (warp == 0 && lane == 0) {
    // TMA producer: the weight tiles of the ring's first round go out before waiting for the
    // previous grid
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
    const uint64_t pol_w = SWAP ? policy_evict_first() : policy_evict_last();
    const uint64_t pol_x = SWAP ? policy_evict_last() : policy_evict_first();
    auto load_w = [&](int i, uint8_t* st, uint64_t* bar) {
      const int kx = (kb0 + i) * KB_ELEMS;
      if (SWAP) {
#pragma unroll
        for (int t = 0; t < NA; ++t) tma_load_2d(st + t * A_BYTES, &tm_w, bar, kx, p0 + t * a.N, pol_w);
      } else {
#pragma unroll
        for (int t = 0; t < NB; ++t) tma_load_2d(st + NA * A_BYTES + t * B_BYTES, &tm_w, bar, kx, q0 + t * a.N, pol_w);
      }
    };
    auto load_x = [&](int i, uint8_t* st, uint64_t* bar) {
      const int kx = (kb0 + i) * KB_ELEMS;
      if (SWAP)
        tma_load_2d(st + NA * A_BYTES, &tm_x, bar, kx, q0, pol_x);
      else
        tma_load_2d(st, &tm_x, bar, kx, p0, pol_x);
    };
    // the ring's whole first round of weights, then (once the previous grid is done) its tokens
    const int pre = min(stages, nkb);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], STAGE_BYTES);
      load_w(i, smem + i * STAGE_BYTES, &full[i]);
    }
    grid_dep_wait();
    for (int i = 0; i < pre; ++i) load_x(i, smem + i * STAGE_BYTES, &full[i]);
    for (int i = pre; i < nkb; ++i) {
      const int s = i % stages;
      const uint32_t round = static_cast<uint32_t>(i / stages);
      if (!mbar_wait(&empty[s], (round - 1) & 1u, a.status)) break;
      uint8_t* st = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      load_w(i, st, &full[s]);
      load_x(i, st, &full[s]);
    }
  } else if (warp == 1) {
    // MMA issuer: the whole warp runs the waits (outcomes made warp-uniform), the elected lane
    // issues and commits
    for (int i = 0; i < nkb; ++i) {
      const int s = i % stages;
      const uint32_t round = static_cast<uint32_t>(i / stages);
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], round & 1u, a.status))) break;
      tc_fence_after();
      const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
      const uint64_t a0 = sw128_desc(base);
      const uint64_t b0 = sw128_desc(base + NA * A_BYTES);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          if (I8)
            mma_i8(tmem, a0 + 2 * k, b0 + 2 * k, IDESC, acc);
          else
            mma_f16(tmem, a0 + 2 * k, b0 + 2 * k, IDESC, acc);
          if (DUAL) {
            const uint64_t a1 = SWAP ? sw128_desc(base + A_BYTES) : a0;
            const uint64_t b1 = SWAP ? b0 : sw128_desc(base + NA * A_BYTES + B_BYTES);
            if (I8)
              mma_i8(tmem + BN, a1 + 2 * k, b1 + 2 * k, IDESC, acc);
            else
              mma_f16(tmem + BN, a1 + 2 * k, b1 + 2 * k, IDESC, acc);
          }
        }
        mma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (elect_one()) mma_commit(accum);
    grid_dep_wait();
  } else {
    grid_dep_wait();
    if (a.rms_ss && warp >= 2) {
      // the tokens' RMSNorm scales, while the MMAs run (the producer's statistics are complete
      // once the previous grid is)
      const int count = SWAP ? BN : 128;
      for (int i = threadIdx.x - 64; i < count; i += kTileThreads - 64)
        rtab_s[i] = rbase + i < a.M ? rms_scale(a, rbase + i) : 1.f;
    }
  }
  __syncwarp();

  // ---------------- epilogue: thread t owns TMEM lane tl = t % 128 (P index p0 + tl) and the
  // 16-column chunks of parity hh = t / 128
  mbar_wait(accum, 0, a.status);
  tc_fence_after();
  const int t = threadIdx.x, tl = t & 127, hh = t >> 7;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  const int p = p0 + tl;
  const float* rtab = nullptr;
  if (a.rms_ss) {
    __syncthreads();  // rtab_s, written by warps 2-3 during the main loop
    rtab = rtab_s;
  }
  float v[16], u[16];
  if (a.splits == 1) {
#pragma unroll 1
    for (int c = hh * 16; c < BN; c += 32) {
      uint32_t r0[16], r1[16];
      tmem_ld16(lane_addr + c, r0);
      if (DUAL) tmem_ld16(lane_addr + BN + c, r1);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[j] = acc_value<I8>(r0[j]);
        u[j] = DUAL ? acc_value<I8>(r1[j]) : 0.f;
      }
      epilogue16<SWAP, DUAL, I8>(a, p, q0 + c, v, u, rtab, rbase);
    }
  } else if (a.cluster_reduce) {
    // stage this split's partial (column-major, lane contiguous) in the now idle stage ring
    float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
    for (int c = hh * 16; c < NACC; c += 32) {
      uint32_t r[16];
      tmem_ld16(lane_addr + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(c + j) * 128 + tl] = acc_value<I8>(r[j]);
    }
    cluster_sync();
    // CTA `rank` reduces row quads [rank*32/S, (rank+1)*32/S): per (quad, column) one 16-byte DSMEM
    // load from every split, all in flight before the sum, which runs in split order
    const int S = a.splits;
    const int rank = static_cast<int>(cluster_ctarank());
    const int qlo = rank * 32 / S, qhi = (rank + 1) * 32 / S, nq = qhi - qlo;
    const uint32_t part_addr = smem_u32(part);
    uint32_t peer[kMaxSplitCluster];
#pragma unroll
    for (int s = 0; s < kMaxSplitCluster; ++s) peer[s] = mapa_shared(part_addr, static_cast<uint32_t>(s < S ? s : 0));
    if (SWAP && !I8 && a.vec_ok) {
      // two items per pass, every load (partials, bias, residual) issued before any store: the
      // output may alias the residual, so the compiler could not reorder them itself
      const int total = nq * BN;
      if (a.stat_ss) {
        for (int i = t; i < BN * 32; i += kTileThreads) stat_red[i] = 0.f;
        __syncthreads();
      }
      for (int base = 0; base < total; base += 2 * kTileThreads) {
        float4 pv[2][kMaxSplitCluster], pu[2][DUAL ? kMaxSplitCluster : 1], bia[2], res[2];
        int ok[2], col[2], quad[2];
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const int idx = base + it * kTileThreads + t;
          ok[it] = idx < total;
          quad[it] = qlo + (ok[it] ? idx % nq : 0);
          col[it] = ok[it] ? idx / nq : 0;
          const int m = q0 + col[it], n = p0 + quad[it] * 4;
          ok[it] = ok[it] && m < a.M && n < a.N;
          const uint32_t off = static_cast<uint32_t>((col[it] * 128 + quad[it] * 4) * 4);
          const uint32_t off_u = static_cast<uint32_t>(((BN + col[it]) * 128 + quad[it] * 4) * 4);
#pragma unroll
          for (int sp = 0; sp < kMaxSplitCluster; ++sp) {
            if (sp < S && ok[it]) {  // padding tokens and features: nothing to load
              pv[it][sp] = ld_cluster_f32x4(peer[sp] + off);
              if constexpr (DUAL) pu[it][sp] = ld_cluster_f32x4(peer[sp] + off_u);
            }
          }
          bia[it] = make_float4(0.f, 0.f, 0.f, 0.f);
          res[it] = bia[it];
          if (ok[it] && n + 4 <= a.N) {
            if (a.bias) bia[it] = __ldg(reinterpret_cast<const float4*>(a.bias + n));
            if (a.res && a.r_type == SO101_F32)
              res[it] = *reinterpret_cast<const float4*>(static_cast<const float*>(a.res) +
                                                        (a.r_period > 0 ? m % a.r_period : out_row(a, m)) * a.ldr + n);
          }
        }
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          if (!ok[it]) continue;
          float4 sv = make_float4(0.f, 0.f, 0.f, 0.f), su = sv;
#pragma unroll
          for (int sp = 0; sp < kMaxSplitCluster; ++sp) {
            if (sp < S) {
              sv.x += pv[it][sp].x, sv.y += pv[it][sp].y, sv.z += pv[it][sp].z, sv.w += pv[it][sp].w;
              if constexpr (DUAL) su.x += pu[it][sp].x, su.y += pu[it][sp].y, su.z += pu[it][sp].z, su.w += pu[it][sp].w;
            }
          }
          if (rtab) {  // the token's RMSNorm scale
            const float rs = rtab[col[it]];
            sv.x *= rs, sv.y *= rs, sv.z *= rs, sv.w *= rs;
            su.x *= rs, su.y *= rs, su.z *= rs, su.w *= rs;
          }
          const int m = q0 + col[it], n = p0 + quad[it] * 4;
          if (n + 4 > a.N || (a.res && a.r_type != SO101_F32) || a.epilogue == SO101_EPI_GELU) {
            const float vv[4] = {sv.x, sv.y, sv.z, sv.w}, uu[4] = {su.x, su.y, su.z, su.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) epilogue1<DUAL, I8>(a, m, n + e, vv[e], uu[e]);
            continue;
          }
          float4 x;
          if constexpr (DUAL) {
            x = make_float4(silu(sv.x) * su.x * a.out_scale, silu(sv.y) * su.y * a.out_scale,
                            silu(sv.z) * su.z * a.out_scale, silu(sv.w) * su.w * a.out_scale);
          } else {
            x = make_float4((sv.x + bia[it].x) * a.out_scale + res[it].x, (sv.y + bia[it].y) * a.out_scale + res[it].y,
                            (sv.z + bia[it].z) * a.out_scale + res[it].z, (sv.w + bia[it].w) * a.out_scale + res[it].w);
          }
          const long long yi = out_row(a, m) * a.ldy + n;
          if (a.y_type == SO101_F32) {
            *reinterpret_cast<float4*>(static_cast<float*>(a.y) + yi) = x;
          } else if (a.y_type == SO101_BF16) {
            __nv_bfloat162 h[2] = {__floats2bfloat162_rn(x.x, x.y), __floats2bfloat162_rn(x.z, x.w)};
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.y) + yi) = *reinterpret_cast<uint2*>(h);
          } else {
            const float vv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              static_cast<int8_t*>(a.y)[yi + e] = static_cast<int8_t>(quant_i8_int(vv[e], a.y_qscale, a.y_qinv));
          }
          if (a.y16) {
            const float4 c = a.y16_scale ? __ldg(reinterpret_cast<const float4*>(a.y16_scale + n))
                                         : make_float4(1.f, 1.f, 1.f, 1.f);
            __nv_bfloat162 h[2] = {__floats2bfloat162_rn(x.x * c.x, x.y * c.y),
                                   __floats2bfloat162_rn(x.z * c.z, x.w * c.w)};
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.y16) + out_row(a, m) * a.ld16 + n) =
                *reinterpret_cast<uint2*>(h);
          }
          if (a.stat_ss) stat_red[col[it] * 32 + quad[it] - qlo] = (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
        }
      }
      if (a.stat_ss) {
        // this rank's feature quads summed per token, in quad order: slot p_tile * S + rank
        __syncthreads();
        if (t < BN && q0 + t < a.M) {
          float sum = 0.f;
          for (int qq = 0; qq < nq; ++qq) sum += stat_red[t * 32 + qq];
          a.stat_ss[static_cast<long long>(q0 + t) * a.stat_ld + p_tile * S + rank] = sum;
        }
      }
    } else {
      for (int idx = t; idx < nq * BN; idx += kTileThreads) {
        const int quad = qlo + idx % nq, col = idx / nq;
        const uint32_t off = static_cast<uint32_t>((col * 128 + quad * 4) * 4);
        const uint32_t off_u = static_cast<uint32_t>(((BN + col) * 128 + quad * 4) * 4);
        float4 pv[kMaxSplitCluster], pu[kMaxSplitCluster];
#pragma unroll
        for (int sp = 0; sp < kMaxSplitCluster; ++sp) {
          if (sp < S) {
            pv[sp] = ld_cluster_f32x4(peer[sp] + off);
            if (DUAL) pu[sp] = ld_cluster_f32x4(peer[sp] + off_u);
          }
        }
        float4 sv = make_float4(0.f, 0.f, 0.f, 0.f), su = sv;
#pragma unroll
        for (int sp = 0; sp < kMaxSplitCluster; ++sp) {
          if (sp < S) {
            sv.x += pv[sp].x, sv.y += pv[sp].y, sv.z += pv[sp].z, sv.w += pv[sp].w;
            if (DUAL) su.x += pu[sp].x, su.y += pu[sp].y, su.z += pu[sp].z, su.w += pu[sp].w;
          }
        }
        const float vv[4] = {sv.x, sv.y, sv.z, sv.w}, uu[4] = {su.x, su.y, su.z, su.w};
        const int qq = q0 + col;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int pp = p0 + quad * 4 + e;
          epilogue1<DUAL, I8>(a, SWAP ? qq : pp, SWAP ? pp : qq, vv[e], uu[e],
                              rtab ? rtab[(SWAP ? qq : pp) - rbase] : 1.f);
        }
      }
    }
    cluster_sync_relaxed();  // no CTA leaves while a peer still reads its shared memory
  } else {
    const int tile = p_tile * a.tiles_q + q_tile;
    uint32_t* ws = static_cast<uint32_t*>(a.ws);
    uint32_t* part = ws + (static_cast<size_t>(tile) * a.splits + split) * NACC * 128;
#pragma unroll 1
    for (int c = hh * 16; c < NACC; c += 32) {
      uint32_t r[16];
      tmem_ld16(lane_addr + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) __stcg(part + (c + j) * 128 + tl, r[j]);
    }
    __threadfence();
    __syncthreads();
    if (t == 0) {
      const int prev = atomicAdd(a.tickets + tile, 1);
      *last_flag = (prev == a.splits - 1);
    }
    __syncthreads();
    if (*last_flag) {
      __threadfence();
      const uint32_t* base = ws + static_cast<size_t>(tile) * a.splits * NACC * 128;
#pragma unroll 1
      for (int c = hh * 16; c < BN; c += 32) {
        if (I8) {
          int iv[16], iu[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) iv[j] = iu[j] = 0;
          for (int s = 0; s < a.splits; ++s) {
            const uint32_t* ps = base + static_cast<size_t>(s) * NACC * 128;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              iv[j] += static_cast<int>(__ldcg(ps + (c + j) * 128 + tl));
              if (DUAL) iu[j] += static_cast<int>(__ldcg(ps + (BN + c + j) * 128 + tl));
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = i32_to_f32(iv[j]);
            u[j] = i32_to_f32(iu[j]);
          }
        } else {
          // all splits' values for 16 columns in flight before the ordered sum
          float pv[16], pu[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = u[j] = 0.f;
          for (int s = 0; s < a.splits; ++s) {
            const uint32_t* ps = base + static_cast<size_t>(s) * NACC * 128;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              pv[j] = __uint_as_float(__ldcg(ps + (c + j) * 128 + tl));
              pu[j] = DUAL ? __uint_as_float(__ldcg(ps + (BN + c + j) * 128 + tl)) : 0.f;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              v[j] += pv[j];
              u[j] += pu[j];
            }
          }
        }
        epilogue16<SWAP, DUAL, I8>(a, p, q0 + c, v, u, rtab, rbase);
      }
      if (t == 0) a.tickets[tile] = 0;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ================================================================ persistent, warp-specialized
constexpr int kEpiWarps = 16;                         // four per SM sub-partition
constexpr int kEpiCols = 256 / (kEpiWarps / 4);       // most columns one epilogue warp owns (BN 256)
constexpr int kBarrierBytes = 256;                    // ring barriers, accumulator barriers, TMEM slot
constexpr int kConstBytes = kEpiWarps * 3 * kEpiCols * 4;  // column constants
// CTA-pair epilogue: per warp a 32-row x 16-column transpose buffer, rows 20 floats apart so that
// both the row-per-lane writes and the column-group reads are free of bank conflicts
constexpr int kOutStride = 20;
constexpr int kOutBytes = kEpiWarps * 32 * kOutStride * 4;

template <int BN, bool DUAL, bool I8>
__global__ void __launch_bounds__(32 * (2 + kEpiWarps), 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                           const GemmArgs a, const int stages) {
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = BN * 128;
  constexpr int NB = DUAL ? 2 : 1;
  constexpr int STAGE_BYTES = A_BYTES + NB * B_BYTES;
  constexpr int NACC = BN * NB;
  constexpr uint32_t TMEM_COLS = 2 * NACC <= 128 ? 128 : 2 * NACC <= 256 ? 256 : 512;
  constexpr uint32_t IDESC = I8 ? idesc_i8(128, BN) : idesc_bf16(128, BN);
  constexpr int KB_ELEMS = I8 ? 128 : 64;
  static_assert(2 * NACC <= 512, "two accumulators must fit in TMEM");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * STAGE_BYTES);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  // per epilogue warp: this tile's column constants (scale, bias, up scale) for its column half
  float* consts = reinterpret_cast<float*>(smem + stages * STAGE_BYTES + kBarrierBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int kb_total = a.kb_total;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      const uint64_t pol_w = policy_evict_last();
      const uint64_t pol_x = policy_evict_first();
      bool waited = false, ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x) {
        const int p0 = (tile / a.tiles_q) * 128, q0 = (tile % a.tiles_q) * BN;
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t round = static_cast<uint32_t>(it / stages);
          if (it >= stages && !mbar_wait(&empty[s], (round - 1) & 1u, a.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          const int kx = kb * KB_ELEMS;
#pragma unroll
          for (int t = 0; t < NB; ++t) tma_load_2d(st + A_BYTES + t * B_BYTES, &tm_w, &full[s], kx, q0 + t * a.N, pol_w);
          if (!waited) {
            grid_dep_wait();
            waited = true;
          }
          tma_load_2d(st, &tm_x, &full[s], kx, p0, pol_x);
        }
      }
      if (!waited) grid_dep_wait();
      grid_dep_launch();
    }
  } else if (warp == 1) {
    // MMA issuer. bf16: the whole warp runs the waits (outcomes made warp-uniform) and its elected
    // lane issues and commits, which keeps the descriptors warp-uniform (expert and prefix GEMMs
    // 10-25% faster). int8: lane 0 alone, which measured 2-8% faster for the vision GEMMs, whose
    // dequantizing epilogue is the bound.
    constexpr bool kWarp = !I8;
    auto wait = [&](uint64_t* b, uint32_t parity) {
      const bool ok = mbar_wait(b, parity, a.status);
      return kWarp ? __all_sync(0xffffffffu, ok) : ok;
    };
    auto issuer = [&]() { return kWarp ? elect_one() : true; };
    if (kWarp || lane == 0) {
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < a.num_tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (local >= 2 && !wait(&acc_empty[buf], (use - 1) & 1u)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * NACC);
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t round = static_cast<uint32_t>(it / stages);
          if (!wait(&full[s], round & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t a0 = sw128_desc(base);
          const uint64_t b0 = sw128_desc(base + A_BYTES);
          if (issuer()) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
              if (I8)
                mma_i8(d, a0 + 2 * k, b0 + 2 * k, IDESC, acc);
              else
                mma_f16(d, a0 + 2 * k, b0 + 2 * k, IDESC, acc);
              if (DUAL) {
                const uint64_t b1 = sw128_desc(base + A_BYTES + B_BYTES);
                if (I8)
                  mma_i8(d + BN, a0 + 2 * k, b1 + 2 * k, IDESC, acc);
                else
                  mma_f16(d + BN, a0 + 2 * k, b1 + 2 * k, IDESC, acc);
              }
            }
            mma_commit(&empty[s]);
          }
          if (kWarp) __syncwarp();
        }
        if (issuer()) mma_commit(&acc_full[buf]);
      }
    }
  } else {
    // epilogue warps: warp e reads TMEM lane quadrant warp % 4 and column group e / 4 (COLS
    // columns). It loads its whole slice of the accumulator into registers, hands the TMEM buffer
    // back to the MMA warp, and only then runs the epilogue arithmetic and the stores.
    grid_dep_wait();
    constexpr int G = kEpiWarps / 4;
    constexpr int COLS = BN / G;
    constexpr int CH = COLS / 16;
    static_assert(COLS % 16 == 0 && COLS * NB <= 64, "epilogue slice must fit in registers");
    const int e = warp - 2;
    const int quad = warp & 3;
    const int c_lo = (e / 4) * COLS;
    float* kc = consts + e * 3 * kEpiCols;
    float* kb = kc + kEpiCols;
    float* ku = kb + kEpiCols;
    int local = 0;
    for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x, ++local) {
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      const int p0 = (tile / a.tiles_q) * 128, q0 = (tile % a.tiles_q) * BN;
      const int p = p0 + quad * 32 + lane;
      // this tile's column constants, staged while the MMAs run
      __syncwarp();
      for (int j = lane; j < COLS; j += 32) {
        const int n = q0 + c_lo + j;
        const bool in = n < a.N;
        kc[j] = I8 ? (in ? a.x_scale * __ldg(a.w_scale + n) : 0.f) : 1.f;
        kb[j] = (a.bias && in) ? __ldg(a.bias + n) : 0.f;
        ku[j] = (I8 && DUAL && in) ? a.x_scale * __ldg(a.w_scale + a.N + n) : 1.f;
      }
      __syncwarp();
      // this row's RMSNorm scale (folded norm), from the producer's sums of squares
      const float rs = (a.rms_ss && p < a.M) ? rms_scale(a, p) : 1.f;
      if (!mbar_wait(&acc_full[buf], use & 1u, a.status)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * NACC + c_lo);
      uint32_t r0[CH][16], r1[DUAL ? CH : 1][16];
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        tmem_ld16(taddr + 16 * c, r0[c]);
        if constexpr (DUAL) tmem_ld16(taddr + BN + 16 * c, r1[c]);
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      float ssq = 0.f;  // this row's sum of squares over the warp's columns (statistics output)
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const int q = q0 + c_lo + 16 * c;
        if (a.vec_ok && p < a.M && q + 16 <= a.N) {
          ssq += epilogue_row16_fast<DUAL, I8>(a, p, q, r0[c], r1[DUAL ? c : 0], kc + 16 * c, kb + 16 * c, ku + 16 * c, rs);
        } else {
          float v[16], u[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = acc_value<I8>(r0[c][j]) * rs;
            u[j] = DUAL ? acc_value<I8>(r1[DUAL ? c : 0][j]) * rs : 0.f;
          }
          epilogue16<false, DUAL, I8>(a, p, q, v, u);
        }
      }
      if (a.stat_ss && p < a.M)  // slot: (column tile, column group)
        a.stat_ss[static_cast<long long>(p) * a.stat_ld + (tile % a.tiles_q) * G + e / 4] = ssq;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ================================================================ CTA pair, persistent
// Two CTAs of a cluster share each 256 x BN output tile (tokens on M). CTA r stages token rows
// [p0 + 128 r, +128) of x and weight rows [q0 + r BN/2, +BN/2) of w in its own shared memory; the
// even CTA issues M = 256 cta_group::2 MMAs over both CTAs' operands, and each CTA's TMEM receives
// its 128 rows x BN columns of the accumulator (two buffers). Per SM that streams 128 x K + BN/2 x K
// operand bytes per 128 x BN outputs instead of 128 x K + BN x K: the large GEMMs are bound by the
// L2 -> SM read rate, not by the tensor pipe. Both CTAs' stage loads complete on the even CTA's
// stage barrier (cta_group::2 TMA), which expects both halves' bytes; commits reach both CTAs'
// barriers (multicast commit); the odd CTA's epilogue warps release a TMEM buffer with remote
// arrives on the even CTA's barrier. Epilogue as the persistent kernel's.
template <int BN, bool DUAL, bool I8>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(32 * (2 + kEpiWarps), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const GemmArgs a, const int stages) {
  constexpr int HB = BN / 2;  // weight rows per CTA
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = HB * 128;
  constexpr int NB = DUAL ? 2 : 1;
  constexpr int STAGE_BYTES = A_BYTES + NB * B_BYTES;
  constexpr int NACC = BN * NB;
  constexpr uint32_t TMEM_COLS = 2 * NACC <= 128 ? 128 : 2 * NACC <= 256 ? 256 : 512;
  constexpr uint32_t IDESC = I8 ? idesc_i8(256, BN) : idesc_bf16(256, BN);
  constexpr int KB_ELEMS = I8 ? 128 : 64;
  static_assert(2 * NACC <= 512, "two accumulators must fit in TMEM");
  static_assert(B_BYTES % 1024 == 0, "swizzled B halves start on 1024-byte boundaries");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + stages * STAGE_BYTES);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2], the even CTA's counts both CTAs' epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  float* consts = reinterpret_cast<float*>(smem + stages * STAGE_BYTES + kBarrierBytes);
  float* stage_out = reinterpret_cast<float*>(smem + stages * STAGE_BYTES + kBarrierBytes + kConstBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);  // used in the even CTA only
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive or multicast commit
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int kb_total = a.kb_total;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_x);
      tma_prefetch_desc(&tm_w);
      const uint64_t pol_w = policy_evict_last();
      const uint64_t pol_x = policy_evict_first();
      bool waited = false, ok = true;
      int it = 0;
      for (int tile = pair; tile < a.num_tiles && ok; tile += npairs) {
        const int p0 = (tile / a.tiles_q) * 256 + static_cast<int>(rank) * 128;
        const int q0 = (tile % a.tiles_q) * BN + static_cast<int>(rank) * HB;
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t round = static_cast<uint32_t>(it / stages);
          if (it >= stages && !mbar_wait(&empty[s], (round - 1) & 1u, a.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
          const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
          const int kx = kb * KB_ELEMS;
#pragma unroll
          for (int t = 0; t < NB; ++t) tma_load_2d_pair(st + A_BYTES + t * B_BYTES, &tm_w, bar, kx, q0 + t * a.N, pol_w);
          if (!waited) {
            grid_dep_wait();
            waited = true;
          }
          tma_load_2d_pair(st, &tm_x, bar, kx, p0, pol_x);
        }
      }
      if (!waited) grid_dep_wait();
      grid_dep_launch();
      // every commit the even CTA sends to this CTA's stage barriers has landed before exit
      for (int j = it - stages; j < it && ok; ++j) {
        if (j < 0) continue;
        ok = mbar_wait(&empty[j % stages], static_cast<uint32_t>(j / stages) & 1u, a.status);
      }
    }
  } else if (warp == 1) {
    // MMA issuer (the even CTA): the whole warp runs the waits (outcomes made warp-uniform), the
    // elected lane issues and commits
    if (leader) {
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = pair; tile < a.num_tiles && ok; tile += npairs, ++local) {
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (local >= 2 && !__all_sync(0xffffffffu, mbar_wait(&acc_empty[buf], (use - 1) & 1u, a.status))) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * NACC);
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t round = static_cast<uint32_t>(it / stages);
          if (!__all_sync(0xffffffffu, mbar_wait(&full[s], round & 1u, a.status))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
          const uint64_t a0 = sw128_desc(base);
          const uint64_t b0 = sw128_desc(base + A_BYTES);
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
              if (I8)
                mma_i8_pair(d, a0 + 2 * k, b0 + 2 * k, IDESC, acc);
              else
                mma_f16_pair(d, a0 + 2 * k, b0 + 2 * k, IDESC, acc);
              if (DUAL) {
                const uint64_t b1 = sw128_desc(base + A_BYTES + B_BYTES);
                if (I8)
                  mma_i8_pair(d + BN, a0 + 2 * k, b1 + 2 * k, IDESC, acc);
                else
                  mma_f16_pair(d + BN, a0 + 2 * k, b1 + 2 * k, IDESC, acc);
              }
            }
            mma_commit_pair(&empty[s]);
          }
          __syncwarp();
        }
        if (ok && elect_one()) mma_commit_pair(&acc_full[buf]);
      }
    }
  } else {
    grid_dep_wait();
    constexpr int G = kEpiWarps / 4;
    constexpr int COLS = BN / G;
    constexpr int CH = COLS / 16;
    static_assert(COLS % 16 == 0 && COLS * NB <= 64, "epilogue slice must fit in registers");
    const int e = warp - 2;
    const int quad = warp & 3;
    const int c_lo = (e / 4) * COLS;
    float* kc = consts + e * 3 * kEpiCols;
    float* kb = kc + kEpiCols;
    float* ku = kb + kEpiCols;
    const uint32_t release_addr = mapa_shared(smem_u32(acc_empty), 0);
    int local = 0;
    for (int tile = pair; tile < a.num_tiles; tile += npairs, ++local) {
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      const int p0 = (tile / a.tiles_q) * 256 + static_cast<int>(rank) * 128, q0 = (tile % a.tiles_q) * BN;
      const int p = p0 + quad * 32 + lane;
      __syncwarp();
      for (int j = lane; j < COLS; j += 32) {
        const int n = q0 + c_lo + j;
        const bool in = n < a.N;
        kc[j] = I8 ? (in ? a.x_scale * __ldg(a.w_scale + n) : 0.f) : 1.f;
        kb[j] = (a.bias && in) ? __ldg(a.bias + n) : 0.f;
        ku[j] = (I8 && DUAL && in) ? a.x_scale * __ldg(a.w_scale + a.N + n) : 1.f;
      }
      __syncwarp();
      const float rs = (a.rms_ss && p < a.M) ? rms_scale(a, p) : 1.f;
      if (!mbar_wait(&acc_full[buf], use & 1u, a.status)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(buf * NACC + c_lo);
      // Accumulator chunk by chunk (16 columns; the next chunk's TMEM load in flight while this one
      // is processed); the buffer goes back to the MMA warp once its last chunk is in registers.
      // Values per row (lane); stores either per row (one 16-byte piece of 32 rows: plain int8
      // output) or through the warp's transpose buffer, each store covering 8 rows x 16 columns
      // (lanes 8 apart share a row): fp32 / bf16 outputs, residuals and bf16 copies.
      const bool transpose = a.y_type != SO101_I8 || a.res || a.y16 || a.stat_ss;
      float* wb = stage_out + e * 32 * kOutStride;
      const int prow0 = p0 + quad * 32, c4 = lane >> 3;
      float ssq4[4] = {0.f, 0.f, 0.f, 0.f};
      float ssq = 0.f;
      // (SiLU gate: two accumulators per chunk, so no load ahead, to stay within the registers)
      uint32_t ra[16], rb[16];
      tmem_ld16(taddr, ra);
      if constexpr (DUAL) tmem_ld16(taddr + BN, rb);
      tmem_ld_wait(ra, rb);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        uint32_t na[16], nb[16];
        if (c + 1 < CH) {
          if constexpr (!DUAL) tmem_ld16(taddr + 16 * (c + 1), na);
        } else {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(release_addr + static_cast<uint32_t>(buf * 8));
        }
        const int q = q0 + c_lo + 16 * c;
        if (a.vec_ok && q + 16 <= a.N) {
          if (transpose) {
            float v[16];
            epilogue_values16<DUAL, I8>(a, ra, rb, kc + 16 * c, kb + 16 * c, ku + 16 * c, rs, v);
            float4* w4 = reinterpret_cast<float4*>(wb + lane * kOutStride);
#pragma unroll
            for (int j = 0; j < 4; ++j) w4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rl = i * 8 + (lane & 7);
              const float4 x = *reinterpret_cast<const float4*>(wb + rl * kOutStride + c4 * 4);
              if (prow0 + rl < a.M) ssq4[i] += epilogue_store4(a, prow0 + rl, q + c4 * 4, x);
            }
            __syncwarp();
          } else if (p < a.M) {
            ssq += epilogue_row16_fast<DUAL, I8>(a, p, q, ra, rb, kc + 16 * c, kb + 16 * c, ku + 16 * c, rs);
          }
        } else if (p < a.M) {
          float v[16], u[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = acc_value<I8>(ra[j]) * rs;
            u[j] = DUAL ? acc_value<I8>(rb[j]) * rs : 0.f;
          }
          epilogue16<false, DUAL, I8>(a, p, q, v, u);
        }
        if (c + 1 < CH) {
          if constexpr (DUAL) {
            tmem_ld16(taddr + 16 * (c + 1), na);
            tmem_ld16(taddr + BN + 16 * (c + 1), nb);
          }
          tmem_ld_wait(na, nb);
#pragma unroll
          for (int j = 0; j < 16; ++j) ra[j] = na[j], rb[j] = nb[j];
        }
      }
      if (a.stat_ss) {  // statistics take the transposed stores
        // row i * 8 + (lane & 7): its four column groups sit in lanes 8 apart
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float t = ssq4[i];
          t += __shfl_xor_sync(0xffffffffu, t, 8);
          t += __shfl_xor_sync(0xffffffffu, t, 16);
          const int m = prow0 + i * 8 + lane;
          if (lane < 8 && m < a.M) a.stat_ss[static_cast<long long>(m) * a.stat_ld + (tile % a.tiles_q) * G + e / 4] = t;
        }
      }
      (void)ssq;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA frees TMEM while the pair's MMAs or epilogues may still use it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, TMEM_COLS);
}

// ============================================================================ host side
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

// 2-D K-major tensor map over rows x inner (elements), row stride ld elements, 128-byte boxes.
int make_map(CUtensorMap* m, const void* ptr, bool i8, long long inner, long long rows, long long ld, int box_rows) {
  EncodeFn enc = encode_fn();
  if (!enc) return SO101_ERR_DRIVER;
  const int esize = i8 ? 1 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SO101_OK : SO101_ERR_ARG;
}

int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

int stage_bytes(int bn, bool swap, bool dual, bool pair = false) {
  const int na = (swap && dual) ? 2 : 1, nb = (!swap && dual) ? 2 : 1;
  return na * 128 * 128 + nb * (pair ? bn / 2 : bn) * 128;
}

constexpr int kSmemBudget = 220 * 1024;
constexpr int kTileScratch = (128 + 64 * 32) * 4;  // tile kernel epilogue scratch: rstd table, statistics
constexpr int kMaxCluster = kMaxSplitCluster;

enum Kind { kTile = 0, kPersistent = 1, kPair = 2 };

struct Plan {
  so101_gemm_config cfg;
  int kind;
  int kb_total, kb_per_split, splits, tiles_p, tiles_q, nacc, cluster;
};

int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

int plan_gemm(int a_type, long long M, long long N, long long K, int epi, const so101_gemm_config* in, Plan* pl) {
  const bool dual = epi == SO101_EPI_SILU_GATE;
  const int kb_elems = a_type == SO101_I8 ? 128 : 64;
  so101_gemm_config c = in ? *in : so101_gemm_config{0, 0, 0, 0, 0};
  so101_gemm_config pick;
  so101_gemm_pick(a_type, M, N, K, epi, &pick);
  if (!in || (c.bn == 0 && c.swap == 0 && c.splits == 0 && c.stages == 0)) {
    const int flags = c.flags;
    c = pick;
    c.flags |= flags;
  }
  if (c.bn == 0) c.bn = pick.bn;
  if (c.splits <= 0) c.splits = 1;
  if (c.swap) {
    if (c.bn != 16 && c.bn != 32 && c.bn != 48 && c.bn != 64) return SO101_ERR_ARG;
    if (a_type == SO101_I8) return SO101_ERR_ARG;
  } else {
    if (c.bn != 64 && c.bn != 128 && c.bn != 192 && c.bn != 256) return SO101_ERR_ARG;
    if (dual && c.bn >= 192) return SO101_ERR_ARG;
  }
  pl->kb_total = ceil_div(K, kb_elems);
  const int splits = c.splits > pl->kb_total ? pl->kb_total : c.splits;
  pl->kb_per_split = ceil_div(pl->kb_total, splits);
  pl->splits = ceil_div(pl->kb_total, pl->kb_per_split);  // no empty split
  c.splits = pl->splits;
  const bool pair = (c.flags & SO101_GEMM_PAIR) && !c.swap && pl->splits == 1 &&
                    (c.bn == 256 || c.bn == 128 || (c.bn == 192 && !dual));
  pl->tiles_p = c.swap ? ceil_div(N, 128) : ceil_div(M, pair ? 256 : 128);
  pl->tiles_q = c.swap ? ceil_div(M, c.bn) : ceil_div(N, c.bn);
  pl->nacc = c.bn * (dual ? 2 : 1);
  const long long tiles = static_cast<long long>(pl->tiles_p) * pl->tiles_q;
  pl->kind = kTile;
  if (pair)
    pl->kind = kPair;
  else if (!c.swap && pl->splits == 1 && !(c.flags & SO101_GEMM_ONE_TILE_PER_CTA) &&
           ((c.flags & SO101_GEMM_PERSISTENT) || tiles >= sm_count()))
    pl->kind = kPersistent;
  if (!pair) c.flags &= ~SO101_GEMM_PAIR;
  if (c.bn == 192 && pl->kind != kPersistent && pl->kind != kPair) return SO101_ERR_ARG;
  pl->cluster = 1;
  if (pl->kind == kTile && pl->splits > 1 && pl->splits <= kMaxCluster && !(c.flags & SO101_GEMM_GLOBAL_SPLITK))
    pl->cluster = pl->splits;
  const bool pers = pl->kind == kPersistent || pl->kind == kPair;
  const int sb = stage_bytes(c.bn, c.swap, dual, pair);
  const int max_st = (kSmemBudget - 1024 - 256 - (pers ? kConstBytes : kTileScratch) - (pair ? kOutBytes : 0)) / sb;
  if (c.stages <= 0) {
    int want = pers ? (pair ? 12 : 8) : pl->kb_per_split;
    if (want < 2) want = 2;
    c.stages = want < max_st ? want : max_st;
    if (c.stages > (pair ? 12 : 8)) c.stages = pair ? 12 : 8;
  }
  if (c.stages < 2 || c.stages > max_st) return SO101_ERR_ARG;
  if (pl->cluster > 1 && c.stages * sb < pl->nacc * 128 * 4) {
    // the cluster reduction stages the partial in the ring: make it big enough
    const int need = ceil_div(static_cast<long long>(pl->nacc) * 512, sb);
    if (need > max_st) return SO101_ERR_ARG;
    c.stages = need;
  }
  pl->cfg = c;
  return SO101_OK;
}

template <typename Kern>
int launch(Kern kern, const CUtensorMap& tx, const CUtensorMap& tw, const GemmArgs& a, dim3 grid, int threads,
           int smem, int cluster, int stages, cudaStream_t stream, bool pdl, int* configured) {
  if (*configured == 0) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return launch_error(e);
    *configured = 1;
  }
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = dim3(threads, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = cluster;
    ++n;
  }
  lc.attrs = attr;
  lc.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kern, tx, tw, a, stages);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}

template <int BN, bool SWAP, bool DUAL, bool I8>
int launch_tile(const CUtensorMap& tx, const CUtensorMap& tw, const GemmArgs& a, const Plan& pl, cudaStream_t stream,
                bool pdl) {
  static int configured = 0;
  const int smem = pl.cfg.stages * stage_bytes(BN, SWAP, DUAL) + 1024 + 256 + kTileScratch;
  return launch(gemm_tc_kernel<BN, SWAP, DUAL, I8>, tx, tw, a, dim3(pl.tiles_q, pl.tiles_p, pl.splits), kTileThreads, smem,
                pl.cluster, pl.cfg.stages, stream, pdl, &configured);
}

template <int BN, bool DUAL, bool I8>
int launch_persistent(const CUtensorMap& tx, const CUtensorMap& tw, const GemmArgs& a, const Plan& pl,
                      cudaStream_t stream, bool pdl) {
  static int configured = 0;
  const int smem = pl.cfg.stages * stage_bytes(BN, false, DUAL) + 1024 + kBarrierBytes + kConstBytes;
  const long long tiles = static_cast<long long>(pl.tiles_p) * pl.tiles_q;
  const int sms = sm_count();
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  return launch(gemm_persistent_kernel<BN, DUAL, I8>, tx, tw, a, dim3(grid, 1, 1), 32 * (2 + kEpiWarps), smem, 1,
                pl.cfg.stages, stream, pdl, &configured);
}

// One cluster of two CTAs per SM pair, as many clusters as can be resident at once.
template <int BN, bool DUAL, bool I8>
int launch_pair(const CUtensorMap& tx, const CUtensorMap& tw, const GemmArgs& a, const Plan& pl, cudaStream_t stream,
                bool pdl) {
  static int configured = 0;
  static int max_clusters = 0;
  const int smem = pl.cfg.stages * stage_bytes(BN, false, DUAL, true) + 1024 + kBarrierBytes + kConstBytes + kOutBytes;
  auto kern = gemm_pair_kernel<BN, DUAL, I8>;
  if (configured == 0) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
    if (e != cudaSuccess) return launch_error(e);
    configured = 1;
  }
  if (max_clusters == 0) {
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
    q.blockDim = dim3(32 * (2 + kEpiWarps), 1, 1);
    q.dynamicSmemBytes = kSmemBudget;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n < 1) n = sm_count() / 2;
    max_clusters = n;
  }
  const long long tiles = static_cast<long long>(pl.tiles_p) * pl.tiles_q;
  const int pairs = static_cast<int>(tiles < max_clusters ? tiles : max_clusters);
  return launch(kern, tx, tw, a, dim3(2 * pairs, 1, 1), 32 * (2 + kEpiWarps), smem, 1, pl.cfg.stages, stream, pdl,
                &configured);
}

template <bool SWAP, bool DUAL, bool I8>
int launch_bn(const CUtensorMap& tx, const CUtensorMap& tw, const GemmArgs& a, const Plan& pl, cudaStream_t stream,
              bool pdl) {
  if constexpr (SWAP) {
    switch (pl.cfg.bn) {
      case 16: return launch_tile<16, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      case 32: return launch_tile<32, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      case 48: return launch_tile<48, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      case 64: return launch_tile<64, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
    }
  } else {
    const bool pers = pl.kind == kPersistent;
    if (pl.kind == kPair) {
      if (pl.cfg.bn == 128) return launch_pair<128, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      if constexpr (!DUAL) {
        if (pl.cfg.bn == 256) return launch_pair<256, DUAL, I8>(tx, tw, a, pl, stream, pdl);
        // N = 720 in four 256 x 192 tiles: 52 pairs on 104 SMs, 224 operand rows per SM
        if (pl.cfg.bn == 192) return launch_pair<192, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      }
      return SO101_ERR_ARG;
    }
    switch (pl.cfg.bn) {
      case 64:
        return pers ? launch_persistent<64, DUAL, I8>(tx, tw, a, pl, stream, pdl)
                    : launch_tile<64, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      case 128:
        return pers ? launch_persistent<128, DUAL, I8>(tx, tw, a, pl, stream, pdl)
                    : launch_tile<128, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
      case 192:  // persistent only: N = 720 in four tiles, 48 columns per epilogue warp
        if constexpr (!DUAL)
          if (pers) return launch_persistent<192, DUAL, I8>(tx, tw, a, pl, stream, pdl);
        break;
      case 256:
        if constexpr (!DUAL)
          return pers ? launch_persistent<256, DUAL, I8>(tx, tw, a, pl, stream, pdl)
                      : launch_tile<256, SWAP, DUAL, I8>(tx, tw, a, pl, stream, pdl);
        break;
    }
  }
  return SO101_ERR_ARG;
}

}  // namespace
}  // namespace so101

using namespace so101;

extern "C" int so101_gemm_pick(int a_type, int64_t M, int64_t N, int64_t K, int epilogue, so101_gemm_config* cfg) {
  if (!cfg) return SO101_ERR_ARG;
  const bool dual = epilogue == SO101_EPI_SILU_GATE;
  const int kb_elems = a_type == SO101_I8 ? 128 : 64;
  const int kb = static_cast<int>((K + kb_elems - 1) / kb_elems);
  const int sms = sm_count();
  so101_gemm_config c = {0, 0, 1, 0, 0};
  if (M <= 64 && a_type == SO101_BF16) {
    // weight streaming: one 128-row weight slab per CTA, K split across a cluster to fill the GPU.
    // More than 32 rows go in two 32-token tiles: each CTA then reduces half the split-K partials
    // (the reduction through distributed shared memory bounds these GEMMs), and the second token
    // tile re-reads its weight slab from L2.
    c.swap = 1;
    c.bn = M <= 16 ? 16 : 32;
    const int tiles = static_cast<int>((N + 127) / 128) * static_cast<int>((M + c.bn - 1) / c.bn);
    int s = sms / tiles;
    if (s > kMaxCluster) s = kMaxCluster;
    const int max_s = kb / 3 > 0 ? kb / 3 : 1;  // at least three K blocks per split
    c.splits = s < 1 ? 1 : (s > max_s ? max_s : s);
  } else if (M <= 256 && a_type == SO101_BF16 && !dual) {
    // a few hundred rows (the prefix at batch 1): still weight streaming, tokens in 64-row tiles
    // on MMA N, so each weight slab is read from HBM once and from L2 by the other token tiles
    c.swap = 1;
    c.bn = 64;
    c.splits = kb >= 8 ? 4 : (kb >= 4 ? 2 : 1);
  } else if (M <= 256 && a_type == SO101_BF16) {
    c.swap = 0;
    c.bn = 64;
    c.splits = 1;
  } else {
    c.swap = 0;
    // 256-wide tiles halve the A-operand shared-memory reads per MMA (128 x 128 tiles need the
    // full shared-memory bandwidth); take them whenever they still give every SM a tile.
    const long long tiles256 = ((M + 127) / 128) * ((N + 255) / 256);
    c.bn = (!dual && (N >= 1024 || (N >= 512 && tiles256 >= sms))) ? 256 : 128;
    if (N <= 128) c.bn = 64;
    const long long tiles = ((M + 127) / 128) * ((N + c.bn - 1) / c.bn);
    c.splits = 1;
    if (tiles < sms / 2) {
      int s = static_cast<int>(sms / tiles);
      const int max_s = kb / 4 > 0 ? kb / 4 : 1;
      c.splits = s > max_s ? max_s : s;
      if (c.splits > kMaxCluster) c.splits = kMaxCluster;
    }
  }
  c.stages = 0;  // chosen by the plan from the problem and the kernel kind
  *cfg = c;
  return SO101_OK;
}

extern "C" int so101_gemm_workspace(int a_type, int64_t M, int64_t N, int64_t K, int epilogue,
                                    const so101_gemm_config* cfg, int64_t* workspace_bytes, int64_t* n_tickets) {
  Plan pl;
  const int rc = plan_gemm(a_type, M, N, K, epilogue, cfg, &pl);
  if (rc) return rc;
  const long long tiles = static_cast<long long>(pl.tiles_p) * pl.tiles_q;
  const bool global = pl.splits > 1 && pl.cluster == 1;
  if (workspace_bytes) *workspace_bytes = global ? tiles * pl.splits * pl.nacc * 128 * 4 : 0;
  if (n_tickets) *n_tickets = global ? tiles : 0;
  return SO101_OK;
}

// Statistics slots a producer plan writes (sums of squares over disjoint feature ranges per row),
// or 0 when the plan cannot produce them: the cluster-reduced swap tiles (one slot per weight tile
// and split) and the persistent kernel (one per column tile and epilogue column group).
int stat_slots_of(const Plan& pl, bool dual, int a_type, long long N) {
  if (dual || a_type != SO101_BF16) return 0;
  if (pl.kind == kPersistent || pl.kind == kPair) return N % 16 == 0 ? pl.tiles_q * (kEpiWarps / 4) : 0;
  if (pl.cfg.swap && pl.cluster > 1 && N % 4 == 0) return pl.tiles_p * pl.splits;
  return 0;
}

extern "C" int so101_gemm_stat_slots(int a_type, int64_t M, int64_t N, int64_t K, int epilogue,
                                     const so101_gemm_config* cfg, int* slots) {
  if (!slots || M <= 0 || N <= 0 || K <= 0) return SO101_ERR_ARG;
  Plan pl;
  const int rc = plan_gemm(a_type, M, N, K, epilogue, cfg, &pl);
  if (rc) return rc;
  *slots = stat_slots_of(pl, epilogue == SO101_EPI_SILU_GATE, a_type, N);
  return *slots > 0 ? SO101_OK : SO101_ERR_ARG;
}

extern "C" int so101_gemm(int a_type, const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy,
                          int y_type, int64_t M, int64_t N, int64_t K, const so101_epilogue* epi,
                          const so101_gemm_config* cfg, void* workspace, int64_t workspace_bytes, int* tickets,
                          int64_t n_tickets, cudaStream_t stream) {
  if (!x || !w || !y || !epi) return SO101_ERR_ARG;
  if (a_type != SO101_BF16 && a_type != SO101_I8) return SO101_ERR_ARG;
  if (M <= 0 || N <= 0 || K <= 0) return SO101_ERR_ARG;
  if (M > (1LL << 30) || N > (1LL << 24) || K > (1LL << 24)) return SO101_ERR_ARG;
  const int esize = a_type == SO101_I8 ? 1 : 2;
  if ((K * esize) % 16 || (ldx * esize) % 16 || (ldw * esize) % 16) return SO101_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16) return SO101_ERR_ARG;
  if (ldx < K || ldw < K) return SO101_ERR_ARG;
  if (y_type != SO101_BF16 && y_type != SO101_F32 && y_type != SO101_I8) return SO101_ERR_ARG;
  if (epi->epilogue < 0 || epi->epilogue > 2) return SO101_ERR_ARG;
  const bool dual = epi->epilogue == SO101_EPI_SILU_GATE;
  if (a_type == SO101_I8 && !epi->w_scale) return SO101_ERR_ARG;
  if (y_type == SO101_I8 && !(epi->y_qscale > 0.f)) return SO101_ERR_ARG;
  if (ldy < N && epi->row_group <= 0) return SO101_ERR_ARG;
  Plan pl;
  int rc = plan_gemm(a_type, M, N, K, epi->epilogue, cfg, &pl);
  if (rc) return rc;
  const long long tiles = static_cast<long long>(pl.tiles_p) * pl.tiles_q;
  if (pl.splits > 1 && pl.cluster == 1) {
    if (!workspace || !tickets || n_tickets < tiles || workspace_bytes < tiles * pl.splits * pl.nacc * 128 * 4)
      return SO101_ERR_WORKSPACE;
  }
  if (pl.tiles_q > 65535 || pl.tiles_p > 65535 || tiles > 0x7fffffffLL) return SO101_ERR_ARG;
  GemmArgs a = {};
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.kb_total = pl.kb_total;
  a.kb_per_split = pl.kb_per_split;
  a.splits = pl.splits;
  a.tiles_q = pl.tiles_q;
  a.num_tiles = static_cast<int>(tiles);
  a.y = y;
  a.ldy = ldy;
  a.y_type = y_type;
  a.epilogue = epi->epilogue;
  a.bias = epi->bias;
  a.res = epi->residual;
  a.ldr = epi->ldr;
  a.r_type = epi->r_type;
  a.r_period = epi->r_period;
  a.out_scale = epi->out_scale == 0.f ? 1.f : epi->out_scale;
  a.w_scale = epi->w_scale;
  a.x_scale = epi->x_scale;
  a.y_qscale = epi->y_qscale;
  a.y_qinv = epi->y_qscale > 0.f ? static_cast<float>(1.0 / static_cast<double>(epi->y_qscale)) : 0.f;
  a.row_group = epi->row_group;
  a.row_stride = epi->row_stride;
  a.ws = workspace;
  a.tickets = tickets;
  a.cluster_reduce = pl.cluster > 1 ? 1 : 0;
  a.status = status_ptr();
  a.rms_ss = epi->rms_ss;
  a.rms_slots = epi->rms_slots;
  a.rms_ld = epi->rms_ld;
  a.rms_n = epi->rms_n;
  a.rms_eps = epi->rms_eps;
  a.stat_ss = epi->stat_ss;
  a.stat_ld = epi->stat_ld;
  a.y16 = epi->y16;
  a.ld16 = epi->ld16;
  a.y16_scale = epi->y16 ? epi->y16_scale : nullptr;
  if (a.y16_scale && reinterpret_cast<uintptr_t>(a.y16_scale) % 16) return SO101_ERR_ARG;
  if (a.rms_ss && (a.rms_slots < 1 || a.rms_slots > 64 || a.rms_ld < a.rms_slots || a.rms_ld % 4 ||
                   reinterpret_cast<uintptr_t>(a.rms_ss) % 16 || !(a.rms_n > 0.f)))
    return SO101_ERR_ARG;
  if (a.stat_ss || a.y16) {
    // statistics and the bf16 copy come from the vectorised epilogues only
    if (a.stat_ss && (stat_slots_of(pl, dual, a_type, N) == 0 || a.stat_ld < stat_slots_of(pl, dual, a_type, N)))
      return SO101_ERR_ARG;
    if (a.y16 && (reinterpret_cast<uintptr_t>(a.y16) % 16 || a.ld16 % 8 || a.ld16 < N || N % 16)) return SO101_ERR_ARG;
    if (epi->epilogue == SO101_EPI_GELU || (a.res && a.r_type != SO101_F32)) return SO101_ERR_ARG;
    if (!pl.cfg.swap && pl.kind != kPersistent && pl.kind != kPair) return SO101_ERR_ARG;
  }
  const int ysz = y_type == SO101_F32 ? 4 : y_type == SO101_BF16 ? 2 : 1;
  bool vec = reinterpret_cast<uintptr_t>(y) % 16 == 0 && (ldy * ysz) % 16 == 0;
  if (a.row_group > 0) vec = vec && (a.row_stride * ldy * ysz) % 16 == 0;
  if (a.res) {
    const int rsz = a.r_type == SO101_F32 ? 4 : 2;
    vec = vec && reinterpret_cast<uintptr_t>(a.res) % 16 == 0 && (a.ldr * rsz) % 16 == 0;
  }
  a.vec_ok = vec ? 1 : 0;
  if ((a.stat_ss || a.y16) && !vec) return SO101_ERR_ARG;

  const bool i8 = a_type == SO101_I8;
  const long long w_rows = dual ? 2 * N : N;
  CUtensorMap tx, tw;
  const int x_box = pl.cfg.swap ? pl.cfg.bn : 128;
  const int w_box = pl.cfg.swap ? 128 : (pl.kind == kPair ? pl.cfg.bn / 2 : pl.cfg.bn);
  rc = make_map(&tx, x, i8, K, M, ldx, x_box);
  if (rc) return rc;
  rc = make_map(&tw, w, i8, K, w_rows, ldw, w_box);
  if (rc) return rc;
  const bool pdl = pdl_enabled();
  if (pl.cfg.swap) {
    if (dual) return launch_bn<true, true, false>(tx, tw, a, pl, stream, pdl);
    return launch_bn<true, false, false>(tx, tw, a, pl, stream, pdl);
  }
  if (i8) {
    if (dual) return SO101_ERR_ARG;
    return launch_bn<false, false, true>(tx, tw, a, pl, stream, pdl);
  }
  if (dual) return launch_bn<false, true, false>(tx, tw, a, pl, stream, pdl);
  return launch_bn<false, false, false>(tx, tw, a, pl, stream, pdl);
}

// ============================================================================ allocation-free entry
// so101_gemm_static: so101_gemm with its split-K scratch (fp32/int32 partials and the ticket
// counters) held in a file-scope device array instead of a caller-allocated workspace. It is for
// callers that cannot allocate device memory: a host stuck inside CUDA-graph capture, a real-time
// control loop that forbids allocation after start-up, or a foreign-language runtime whose only
// handle on the GPU is this library. Every GPU that loads the library holds the array until the
// process exits.
namespace so101 {
namespace {

constexpr long long kStaticPartialBytes = 8ll << 20;  // 8 MiB of split-K partials
constexpr long long kStaticTickets = 4096;            // one per output tile

static __device__ __align__(256) unsigned char g_static_scratch[kStaticPartialBytes + kStaticTickets * 4];

// Host-side device address of g_static_scratch, looked up per device with that device current
// (the symbol's host name is only a stand-in, never a device address). The address belongs to the
// device's current context: it is kept beside that context's handle and looked up again when the
// context changes (after cudaDeviceReset a new primary context loads the module afresh).
struct StaticScratch {
  void* ctx = nullptr;
  void* base = nullptr;
};
StaticScratch g_static_scratch_addr[64];
std::mutex g_static_scratch_mu;

using CtxGetCurrentFn = int (*)(void**);  // CUresult cuCtxGetCurrent(CUcontext*)

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  return fn;
}

int static_scratch(void** partials, int** tickets) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SO101_ERR_LAUNCH;
  CtxGetCurrentFn get = ctx_get_current();
  void* ctx = nullptr;  // null before the runtime's first call on this thread made a context current
  if (!get || get(&ctx) != 0) return SO101_ERR_DRIVER;
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  StaticScratch& slot = g_static_scratch_addr[dev];
  if (!ctx || !slot.base || slot.ctx != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || !p) return SO101_ERR_LAUNCH;
    if (get(&ctx) != 0 || !ctx) return SO101_ERR_LAUNCH;
    slot.base = p;
    slot.ctx = ctx;
  }
  *partials = slot.base;
  *tickets = reinterpret_cast<int*>(static_cast<unsigned char*>(slot.base) + kStaticPartialBytes);
  return SO101_OK;
}

}  // namespace
}  // namespace so101

extern "C" int so101_gemm_static(int a_type, const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
                                 int64_t ldy, int y_type, int64_t M, int64_t N, int64_t K,
                                 const so101_epilogue* epi, const so101_gemm_config* cfg, cudaStream_t stream) {
  if (!epi) return SO101_ERR_ARG;
  int64_t need = 0, tick = 0;
  int rc = so101_gemm_workspace(a_type, M, N, K, epi->epilogue, cfg, &need, &tick);
  if (rc) return rc;
  if (need > so101::kStaticPartialBytes || tick > so101::kStaticTickets) return SO101_ERR_WORKSPACE;
  void* partials = nullptr;
  int* tickets = nullptr;
  rc = so101::static_scratch(&partials, &tickets);
  if (rc) return rc;
  // the tickets must read zero when the kernel starts; a completed call leaves them zero, this
  // also clears what an interrupted one left behind (a stream-ordered memset, not an allocation)
  if (tick > 0 && cudaMemsetAsync(tickets, 0, static_cast<size_t>(tick) * sizeof(int), stream) != cudaSuccess)
    return SO101_ERR_LAUNCH;
  return so101_gemm(a_type, x, ldx, w, ldw, y, ldy, y_type, M, N, K, epi, cfg, partials,
                    so101::kStaticPartialBytes, tickets, so101::kStaticTickets, stream);
}
