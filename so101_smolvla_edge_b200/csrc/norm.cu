// Row-wise kernels: RMSNorm, LayerNorm (+ pixel shuffle, + int8 quantization), RoPE and the K/V
// cache write, absmax calibration and int8 weight packing. One warp per row; all HBM-bound.
#include "common.cuh"

namespace so101 {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float ld_any(const void* p, long long i, int type) {
  return type == SO101_F32 ? static_cast<const float*>(p)[i]
                           : __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void st_any(void* p, long long i, int type, float v, float qs) {
  if (type == SO101_F32)
    static_cast<float*>(p)[i] = v;
  else if (type == SO101_BF16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<int8_t*>(p)[i] = quant_i8(v, qs);
}

constexpr int kMaxRowPerLane = 32;  // rows up to 32 * 32 = 1024 wide stay in registers

// ------------------------------------------------------------------ RMSNorm (one warp per row)
__global__ void rms_norm_kernel(const void* __restrict__ x, long long ldx, int x_type,
                                const float* __restrict__ w, void* __restrict__ y, long long ldy,
                                int y_type, long long rows, int n, float eps) {
  grid_dep_launch();
  grid_dep_wait();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[kMaxRowPerLane];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxRowPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < n ? ld_any(x, row * ldx + c, x_type) : 0.f;
    ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / static_cast<float>(n) + eps);
#pragma unroll
  for (int i = 0; i < kMaxRowPerLane; ++i) {
    const int c = lane + 32 * i;
    if (c < n) st_any(y, row * ldy + c, y_type, (v[i] * rstd) * w[c], 1.f);
  }
}

// ------------------------------------------------------------------ LayerNorm (+ pixel shuffle)
// shuffle > 1: input row r = image * T + (hi * side + wi) goes to output row
// image * T / s^2 + (hi / s) * (side / s) + wi / s, columns ((hi % s) * s + wi % s) * n + c.
__global__ void layer_norm_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w,
                                  const float* __restrict__ b, void* __restrict__ y, long long ldy,
                                  int y_type, float qs, long long rows, int n, float eps, int s,
                                  long long T) {
  grid_dep_launch();
  grid_dep_wait();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[kMaxRowPerLane];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxRowPerLane; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < n ? x[row * ldx + c] : 0.f;
    sum += v[i];
  }
  const float mu = warp_sum(sum) / static_cast<float>(n);
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxRowPerLane; ++i) {
    const int c = lane + 32 * i;
    const float d = c < n ? v[i] - mu : 0.f;
    var += d * d;
  }
  const float rstd = rsqrtf(warp_sum(var) / static_cast<float>(n) + eps);
  long long out_row = row, col0 = 0;
  if (s > 1) {
    const long long img = row / T, tok = row % T;
    const int side = static_cast<int>(sqrtf(static_cast<float>(T)) + 0.5f);
    const int hi = static_cast<int>(tok / side), wi = static_cast<int>(tok % side);
    out_row = img * (T / (s * s)) + (hi / s) * (side / s) + wi / s;
    col0 = static_cast<long long>((hi % s) * s + wi % s) * n;
  }
#pragma unroll
  for (int i = 0; i < kMaxRowPerLane; ++i) {
    const int c = lane + 32 * i;
    if (c < n) st_any(y, out_row * ldy + col0 + c, y_type, (v[i] - mu) * rstd * w[c] + b[c], qs);
  }
}

// ------------------------------------------------------------------ vectorized row kernels
// One warp per row, lane l holding float4 groups l, l + 32, ... (G groups, n <= 128 G, n % 4 == 0,
// 16-byte aligned rows): the row is read once with 16-byte loads and written with packed stores.
__device__ __forceinline__ void store4(void* y, long long i, int type, float a, float b, float c, float d, float inv) {
  if (type == SO101_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(y) + i) = make_float4(a, b, c, d);
  } else if (type == SO101_BF16) {
    __nv_bfloat162 h[2] = {__floats2bfloat162_rn(a, b), __floats2bfloat162_rn(c, d)};
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(y) + i) = *reinterpret_cast<uint2*>(h);
  } else {
    *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(y) + i) = pack4_i8(a, b, c, d, inv);
  }
}

template <int G>
__global__ void layer_norm_vec_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w,
                                      const float* __restrict__ b, void* __restrict__ y, long long ldy, int y_type,
                                      float inv_qs, long long rows, int n, float eps, int s, long long T) {
  grid_dep_launch();
  grid_dep_wait();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * ldx);
  float4 v[G];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int g = lane + 32 * i;
    v[i] = 4 * g < n ? xr[g] : make_float4(0.f, 0.f, 0.f, 0.f);
    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  const float inv_n = 1.0f / static_cast<float>(n);
  const float mu = warp_sum(sum) * inv_n;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < G; ++i) {
    if (4 * (lane + 32 * i) < n) {
      const float a0 = v[i].x - mu, a1 = v[i].y - mu, a2 = v[i].z - mu, a3 = v[i].w - mu;
      var += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
    }
  }
  const float rstd = rsqrtf(warp_sum(var) * inv_n + eps);
  long long orow = row, col0 = 0;
  if (s > 1) {
    const long long img = row / T, tok = row % T;
    const int side = static_cast<int>(sqrtf(static_cast<float>(T)) + 0.5f);
    const int hi = static_cast<int>(tok / side), wi = static_cast<int>(tok % side);
    orow = img * (T / (s * s)) + (hi / s) * (side / s) + wi / s;
    col0 = static_cast<long long>((hi % s) * s + wi % s) * n;
  }
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int c = 4 * (lane + 32 * i);
    if (c >= n) continue;
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w + c));
    const float4 bb = __ldg(reinterpret_cast<const float4*>(b + c));
    store4(y, orow * ldy + col0 + c, y_type, (v[i].x - mu) * rstd * ww.x + bb.x, (v[i].y - mu) * rstd * ww.y + bb.y,
           (v[i].z - mu) * rstd * ww.z + bb.z, (v[i].w - mu) * rstd * ww.w + bb.w, inv_qs);
  }
}

template <int G>
__global__ void rms_norm_vec_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w,
                                    void* __restrict__ y, long long ldy, int y_type, long long rows, int n, float eps) {
  grid_dep_launch();
  grid_dep_wait();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + row * ldx);
  float4 v[G];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int g = lane + 32 * i;
    v[i] = 4 * g < n ? xr[g] : make_float4(0.f, 0.f, 0.f, 0.f);
    ss += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
  }
  const float rstd = rsqrtf(warp_sum(ss) / static_cast<float>(n) + eps);
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int c = 4 * (lane + 32 * i);
    if (c >= n) continue;
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w + c));
    store4(y, row * ldy + c, y_type, (v[i].x * rstd) * ww.x, (v[i].y * rstd) * ww.y, (v[i].z * rstd) * ww.z,
           (v[i].w * rstd) * ww.w, 1.f);
  }
}

// Statistics for an RMSNorm applied in the consuming GEMM: per row, the sum of squares (slot 0 of
// stat_ss, row stride stat_ld) and the bf16 row times the norm weight w (NULL: 1). One warp per row.
__global__ void rms_stats_kernel(const float* __restrict__ x, long long ldx, long long rows, int n,
                                 const float* __restrict__ w, __nv_bfloat16* __restrict__ y16, long long ld16,
                                 float* __restrict__ stat, long long stat_ld) {
  grid_dep_launch();
  grid_dep_wait();
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float ss = 0.f;
  for (int c = 4 * lane; c < n; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(x + row * ldx + c);
    ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
    const float4 sc = w ? __ldg(reinterpret_cast<const float4*>(w + c)) : make_float4(1.f, 1.f, 1.f, 1.f);
    __nv_bfloat162 h[2] = {__floats2bfloat162_rn(v.x * sc.x, v.y * sc.y), __floats2bfloat162_rn(v.z * sc.z, v.w * sc.w)};
    *reinterpret_cast<uint2*>(y16 + row * ld16 + c) = *reinterpret_cast<uint2*>(h);
  }
  ss = warp_sum(ss);
  if (lane == 0) stat[row * stat_ld] = ss;
}

// ------------------------------------------------------------------ RoPE + K/V cache write
// grid (rows, batch); thread j < nkv * hd/2 rotates pair (d, d + hd/2) of kv head j / (hd/2) and
// copies the two value columns at the same positions. The rotation is rounded per operation
// (no FMA contraction), as torch evaluates x1*c - x2*s and x2*c + x1*s.
__global__ void rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, long long ldq, int nq, int nkv,
                               int hd, const float* __restrict__ cos, const float* __restrict__ sin,
                               __nv_bfloat16* __restrict__ k_out, long long ldk,
                               __nv_bfloat16* __restrict__ v_out, long long ldv, long long b_qkv,
                               long long b_k, long long b_v) {
  grid_dep_launch();
  grid_dep_wait();
  const long long r = blockIdx.x;
  const int bi = blockIdx.y;
  const int half = hd / 2;
  const __nv_bfloat16* src = qkv + bi * b_qkv + r * ldq;
  for (int j = threadIdx.x; j < nkv * half; j += blockDim.x) {
    const int h = j / half, d = j % half;
    const float k1 = __bfloat162float(src[(nq + h) * hd + d]);
    const float k2 = __bfloat162float(src[(nq + h) * hd + d + half]);
    const float c = cos[r * half + d], sn = sin[r * half + d];
    __nv_bfloat16* kd = k_out + bi * b_k + r * ldk + h * hd;
    kd[d] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(k1, c), __fmul_rn(k2, sn)));
    kd[d + half] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(k2, c), __fmul_rn(k1, sn)));
    if (v_out) {
      __nv_bfloat16* vd = v_out + bi * b_v + r * ldv + h * hd;
      vd[d] = src[(nq + nkv + h) * hd + d];
      vd[d + half] = src[(nq + nkv + h) * hd + d + half];
    }
  }
}

// ------------------------------------------------------------------ calibration and packing
__global__ void absmax_kernel(const void* __restrict__ x, long long ldx, int x_type, long long rows,
                              long long n, float* amax) {
  grid_dep_launch();
  grid_dep_wait();
  float m = 0.f;
  const long long total = rows * n;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / n, c = i % n;
    m = fmaxf(m, fabsf(ld_any(x, r * ldx + c, x_type)));
  }
  m = warp_max(m);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<int*>(amax), __float_as_int(t));
  }
}

// one block per output channel n
__global__ void quantize_weight_kernel(const void* __restrict__ w, int w_type, long long K,
                                       int8_t* __restrict__ wq, float* __restrict__ scale) {
  grid_dep_launch();
  grid_dep_wait();
  const long long n = blockIdx.x;
  float m = 0.f;
  for (long long k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(ld_any(w, n * K + k, w_type)));
  m = warp_max(m);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = fmaxf(t / 127.0f, 1e-8f);
  }
  __syncthreads();
  const float s = red[0];
  if (threadIdx.x == 0) scale[n] = s;
  for (long long k = threadIdx.x; k < K; k += blockDim.x) {
    float q = rintf(ld_any(w, n * K + k, w_type) / s);
    q = fminf(fmaxf(q, -127.f), 127.f);
    wq[n * K + k] = static_cast<int8_t>(static_cast<int>(q));
  }
}

}  // namespace so101

using namespace so101;


namespace {
bool vec_ok(const void* x, long long ldx, int esz, const void* y, long long ldy, int ysz, const float* w, long long n) {
  return n % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && (ldx * esz) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(y) % 16 == 0 && (ldy * ysz) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0;
}
}  // namespace

extern "C" int so101_rms_norm(const void* x, int64_t ldx, int x_type, const float* w, void* y, int64_t ldy,
                              int y_type, int64_t rows, int64_t n, float eps, cudaStream_t stream) {
  if (!x || !w || !y || rows <= 0 || n <= 0 || n > 32 * kMaxRowPerLane) return SO101_ERR_ARG;
  if (x_type != SO101_F32 && x_type != SO101_BF16) return SO101_ERR_ARG;
  if (y_type != SO101_F32 && y_type != SO101_BF16) return SO101_ERR_ARG;
  const int rows_per_block = 4;
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
  const int ysz = y_type == SO101_F32 ? 4 : 2;
  if (x_type == SO101_F32 && vec_ok(x, ldx, 4, y, ldy, ysz, w, n) && (ldy * ysz) % 16 == 0) {
    const dim3 g(static_cast<unsigned>(blocks)), bl(32 * rows_per_block);
    const float* xf = static_cast<const float*>(x);
    const int ni = static_cast<int>(n);
    switch ((n + 127) / 128) {
      case 1: return launch_kernel(rms_norm_vec_kernel<1>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 2: return launch_kernel(rms_norm_vec_kernel<2>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 3: return launch_kernel(rms_norm_vec_kernel<3>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 4: return launch_kernel(rms_norm_vec_kernel<4>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 5: return launch_kernel(rms_norm_vec_kernel<5>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 6: return launch_kernel(rms_norm_vec_kernel<6>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 7: return launch_kernel(rms_norm_vec_kernel<7>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
      case 8: return launch_kernel(rms_norm_vec_kernel<8>, g, bl, 0, stream, xf, ldx, w, y, ldy, y_type, rows, ni, eps);
    }
  }
  return launch_kernel(rms_norm_kernel, dim3(static_cast<unsigned>(blocks)), dim3(32 * rows_per_block), 0, stream,
                       x, ldx, x_type, w, y, ldy, y_type, rows, static_cast<int>(n), eps);
}

extern "C" int so101_rms_stats(const float* x, int64_t ldx, int64_t rows, int64_t n, const float* w, void* y16,
                               int64_t ld16, float* stat_ss, int64_t stat_ld, cudaStream_t stream) {
  if (!x || !y16 || !stat_ss || rows <= 0 || n <= 0 || n % 4 || n > (1 << 20)) return SO101_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 16 || ldx % 4 || reinterpret_cast<uintptr_t>(y16) % 8 || ld16 % 4 ||
      reinterpret_cast<uintptr_t>(w) % 16 || stat_ld < 1 || ldx < n || ld16 < n)
    return SO101_ERR_ARG;
  const int rows_per_block = 4;
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(rms_stats_kernel, dim3(static_cast<unsigned>(blocks)), dim3(32 * rows_per_block), 0, stream,
                       x, ldx, rows, static_cast<int>(n), w, static_cast<__nv_bfloat16*>(y16), ld16, stat_ss,
                       stat_ld);
}

extern "C" int so101_layer_norm(const float* x, int64_t ldx, const float* w, const float* b, void* y,
                                int64_t ldy, int y_type, float y_qscale, int64_t rows, int64_t n, float eps,
                                int shuffle, int64_t tokens_per_image, cudaStream_t stream) {
  if (!x || !w || !b || !y || rows <= 0 || n <= 0 || n > 32 * kMaxRowPerLane) return SO101_ERR_ARG;
  if (y_type != SO101_BF16 && y_type != SO101_I8 && y_type != SO101_F32) return SO101_ERR_ARG;
  if (y_type == SO101_I8 && !(y_qscale > 0.f)) return SO101_ERR_ARG;
  if (shuffle > 1) {
    const int side = static_cast<int>(sqrt(static_cast<double>(tokens_per_image)) + 0.5);
    if (tokens_per_image <= 0 || static_cast<long long>(side) * side != tokens_per_image || side % shuffle ||
        rows % tokens_per_image)
      return SO101_ERR_ARG;
  }
  const int rows_per_block = 4;
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  const int ysz = y_type == SO101_F32 ? 4 : y_type == SO101_BF16 ? 2 : 1;
  if (vec_ok(x, ldx, 4, y, ldy, ysz, w, n) && reinterpret_cast<uintptr_t>(b) % 16 == 0) {
    const dim3 g(static_cast<unsigned>(blocks)), bl(32 * rows_per_block);
    const float inv = y_type == SO101_I8 ? static_cast<float>(1.0 / static_cast<double>(y_qscale)) : 1.f;
    const int ni = static_cast<int>(n), sh = shuffle > 1 ? shuffle : 1;
    const long long T = shuffle > 1 ? tokens_per_image : 1;
    switch ((n + 127) / 128) {
      case 1: return launch_kernel(layer_norm_vec_kernel<1>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 2: return launch_kernel(layer_norm_vec_kernel<2>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 3: return launch_kernel(layer_norm_vec_kernel<3>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 4: return launch_kernel(layer_norm_vec_kernel<4>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 5: return launch_kernel(layer_norm_vec_kernel<5>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 6: return launch_kernel(layer_norm_vec_kernel<6>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 7: return launch_kernel(layer_norm_vec_kernel<7>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
      case 8: return launch_kernel(layer_norm_vec_kernel<8>, g, bl, 0, stream, x, ldx, w, b, y, ldy, y_type, inv, rows, ni, eps, sh, T);
    }
  }
  return launch_kernel(layer_norm_kernel, dim3(static_cast<unsigned>(blocks)), dim3(32 * rows_per_block), 0, stream,
                       x, ldx, w, b, y, ldy, y_type, y_qscale, rows, static_cast<int>(n), eps, shuffle > 1 ? shuffle : 1,
      shuffle > 1 ? tokens_per_image : 1);
}

extern "C" int so101_rope_kv(const void* qkv, int64_t ldqkv, int nq, int nkv, int hd, const float* cos,
                             const float* sin, void* k_out, int64_t ldk, void* v_out, int64_t ldv, int64_t rows,
                             int batch, int64_t b_qkv, int64_t b_k, int64_t b_v, cudaStream_t stream) {
  if (!qkv || !cos || !sin || !k_out || rows <= 0 || batch <= 0 || hd <= 0 || hd % 2 || nkv <= 0)
    return SO101_ERR_ARG;
  if (rows > 0x7fffffffLL || batch > 65535) return SO101_ERR_ARG;
  const int threads = nkv * hd / 2 < 256 ? ((nkv * hd / 2 + 31) / 32) * 32 : 256;
  return launch_kernel(rope_kv_kernel, dim3(dim3(static_cast<unsigned>(rows), batch)), dim3(threads), 0, stream,
                       static_cast<const __nv_bfloat16*>(qkv), ldqkv, nq, nkv, hd, cos, sin, static_cast<__nv_bfloat16*>(k_out),
      ldk, static_cast<__nv_bfloat16*>(v_out), ldv, b_qkv, b_k, b_v);
}

extern "C" int so101_absmax(const void* x, int64_t ldx, int x_type, int64_t rows, int64_t n, float* amax,
                            cudaStream_t stream) {
  if (!x || !amax || rows <= 0 || n <= 0) return SO101_ERR_ARG;
  if (x_type != SO101_F32 && x_type != SO101_BF16) return SO101_ERR_ARG;
  long long blocks = (rows * n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  return launch_kernel(absmax_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                       x, ldx, x_type, rows, n, amax);
}

extern "C" int so101_quantize_weight(const void* w, int w_type, int64_t N, int64_t K, int8_t* w_q, float* scale,
                                     cudaStream_t stream) {
  if (!w || !w_q || !scale || N <= 0 || K <= 0 || N > 0x7fffffffLL) return SO101_ERR_ARG;
  if (w_type != SO101_F32 && w_type != SO101_BF16) return SO101_ERR_ARG;
  return launch_kernel(quantize_weight_kernel, dim3(static_cast<unsigned>(N)), dim3(256), 0, stream,
                       w, w_type, K, w_q, scale);
}
