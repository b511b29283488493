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


extern "C" int so101_rms_norm(const void* x, int64_t ldx, int x_type, const float* w, void* y, int64_t ldy,
                              int y_type, int64_t rows, int64_t n, float eps, cudaStream_t stream) {
  if (!x || !w || !y || rows <= 0 || n <= 0 || n > 32 * kMaxRowPerLane) return SO101_ERR_ARG;
  if (x_type != SO101_F32 && x_type != SO101_BF16) return SO101_ERR_ARG;
  if (y_type != SO101_F32 && y_type != SO101_BF16) return SO101_ERR_ARG;
  const int rows_per_block = 4;
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(rms_norm_kernel, dim3(static_cast<unsigned>(blocks)), dim3(32 * rows_per_block), 0, stream,
                       x, ldx, x_type, w, y, ldy, y_type, rows, static_cast<int>(n), eps);
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
