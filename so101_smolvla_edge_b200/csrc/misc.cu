// Small kernels around the GEMMs: frame preprocessing into patch rows, fp32 CUDA-core linears
// (the reference keeps the action/time/state MLPs in fp32), the expert's output head fused with
// the Euler step, the prefix tail rows (task tokens + state) and the unnormalisation.
#include "common.cuh"

namespace so101 {

// ------------------------------------------------------------------ preprocess + patch unfold
// One thread per output pair (2 features). Output row = img * G^2 + gy * G + gx, feature =
// c * P * P + py * P + px; pixel (Y, X) = (gy * P + py, gx * P + px) of the padded S x S image.
// Pixels left of S - rw or above S - rh are padding (0 -> -1 after *2-1); the rest are bilinear
// samples (align_corners = False, source index clamped at 0) of the h x w frame scaled to
// rh x rw.
__device__ __forceinline__ float pixel(const uint8_t* __restrict__ img, int h, int w, int c, int yr, int xr,
                                       float sh, float sw) {
  float sy = sh * (static_cast<float>(yr) + 0.5f) - 0.5f;
  float sx = sw * (static_cast<float>(xr) + 0.5f) - 0.5f;
  sy = sy < 0.f ? 0.f : sy;
  sx = sx < 0.f ? 0.f : sx;
  const int y0 = static_cast<int>(sy), x0 = static_cast<int>(sx);
  const int y1 = y0 < h - 1 ? y0 + 1 : y0, x1 = x0 < w - 1 ? x0 + 1 : x0;
  const float ly = sy - static_cast<float>(y0), lx = sx - static_cast<float>(x0);
  const float hy = 1.f - ly, hx = 1.f - lx;
  const float v00 = static_cast<float>(img[(static_cast<long long>(y0) * w + x0) * 3 + c]) / 255.0f;
  const float v01 = static_cast<float>(img[(static_cast<long long>(y0) * w + x1) * 3 + c]) / 255.0f;
  const float v10 = static_cast<float>(img[(static_cast<long long>(y1) * w + x0) * 3 + c]) / 255.0f;
  const float v11 = static_cast<float>(img[(static_cast<long long>(y1) * w + x1) * 3 + c]) / 255.0f;
  return hy * (hx * v00 + lx * v01) + ly * (hx * v10 + lx * v11);
}

__global__ void preprocess_kernel(const uint8_t* __restrict__ img, int n_img, int h, int w, int rh, int rw,
                                  int S, int P, void* __restrict__ out, int y_type, float qs) {
  grid_dep_launch();
  grid_dep_wait();
  const int G = S / P, F = 3 * P * P;
  const long long pairs = static_cast<long long>(n_img) * G * G * (F / 2);
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= pairs) return;
  const long long e = i * 2;
  const long long row = e / F;
  const int f0 = static_cast<int>(e % F);
  const int im = static_cast<int>(row / (G * G));
  const int pr = static_cast<int>(row % (G * G));
  const int gy = pr / G, gx = pr % G;
  const uint8_t* src = img + static_cast<long long>(im) * h * w * 3;
  const float sh = static_cast<float>(h) / static_cast<float>(rh);
  const float sw = static_cast<float>(w) / static_cast<float>(rw);
  float v[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int f = f0 + t;
    const int c = f / (P * P), py = (f / P) % P, px = f % P;
    const int Y = gy * P + py, X = gx * P + px;
    const int yr = Y - (S - rh), xr = X - (S - rw);
    float val = 0.f;
    if (yr >= 0 && xr >= 0) {
      if (rh == h && rw == w)
        val = static_cast<float>(src[(static_cast<long long>(yr) * w + xr) * 3 + c]) / 255.0f;
      else
        val = pixel(src, h, w, c, yr, xr, sh, sw);
    }
    v[t] = val * 2.0f - 1.0f;
  }
  if (y_type == SO101_BF16) {
    reinterpret_cast<__nv_bfloat162*>(out)[i] = __floats2bfloat162_rn(v[0], v[1]);
  } else if (y_type == SO101_I8) {
    int8_t* o = static_cast<int8_t*>(out) + e;
    o[0] = quant_i8(v[0], qs);
    o[1] = quant_i8(v[1], qs);
  } else {
    float* o = static_cast<float*>(out) + e;
    o[0] = v[0];
    o[1] = v[1];
  }
}

// The same for frames already at the model's size (no resize, no padding) and 16 x 16 patches:
// one warp per patch. Its 16 rows of 48 bytes come in as 16-byte loads (each input byte once)
// through shared memory, and its 768 channel-major values leave as 16-byte stores; the per-value
// arithmetic is preprocess_kernel's.
constexpr int kPpWarps = 8;

__global__ void __launch_bounds__(32 * kPpWarps) preprocess_patch_kernel(const uint8_t* __restrict__ img,
                                                                       int n_img, int S, void* __restrict__ out,
                                                                       int y_type, float qs) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ __align__(16) uint8_t tiles[kPpWarps][16 * 48];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = S / 16;
  const long long patch = static_cast<long long>(blockIdx.x) * kPpWarps + warp;
  if (patch >= static_cast<long long>(n_img) * G * G) return;  // whole warps
  const int im = static_cast<int>(patch / (G * G)), pr = static_cast<int>(patch % (G * G));
  const int gy = pr / G, gx = pr % G;
  const uint8_t* src = img + (static_cast<long long>(im) * S * S + static_cast<long long>(gy) * 16 * S + gx * 16) * 3;
  uint8_t* t = tiles[warp];
  for (int c = lane; c < 48; c += 32) {  // row c / 3, 16-byte piece c % 3
    const int r = c / 3, k = c % 3;
    *reinterpret_cast<uint4*>(t + r * 48 + k * 16) =
        __ldg(reinterpret_cast<const uint4*>(src + static_cast<long long>(r) * S * 3 + k * 16));
  }
  __syncwarp();
  auto value = [&](int ch, int py, int px) {
    const float val = static_cast<float>(t[py * 48 + px * 3 + ch]) / 255.0f;
    return val * 2.0f - 1.0f;
  };
  if (y_type == SO101_I8) {
    int8_t* o = static_cast<int8_t*>(out) + patch * 768;
    for (int c = lane; c < 48; c += 32) {  // 16 values: channel c / 16, patch row c % 16
      const int ch = c / 16, py = c % 16;
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t packed = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b)
          packed |= static_cast<uint32_t>(static_cast<uint8_t>(quant_i8(value(ch, py, 4 * q + b), qs))) << (8 * b);
        wv[q] = packed;
      }
      *reinterpret_cast<uint4*>(o + c * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  } else if (y_type == SO101_BF16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out) + patch * 768;
    for (int c = lane; c < 96; c += 32) {  // 8 values: channel c / 32, patch row (c / 2) % 16, half c % 2
      const int ch = c / 32, py = (c / 2) % 16, px0 = (c % 2) * 8;
      __nv_bfloat162 hv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) hv[q] = __floats2bfloat162_rn(value(ch, py, px0 + 2 * q), value(ch, py, px0 + 2 * q + 1));
      *reinterpret_cast<uint4*>(o + c * 8) = *reinterpret_cast<const uint4*>(hv);
    }
  } else {
    float* o = static_cast<float*>(out) + patch * 768;
    for (int c = lane; c < 192; c += 32) {  // 4 values: channel c / 64, patch row (c / 4) % 16, quarter c % 4
      const int ch = c / 64, py = (c / 4) % 16, px0 = (c % 4) * 4;
      *reinterpret_cast<float4*>(o + c * 4) =
          make_float4(value(ch, py, px0), value(ch, py, px0 + 1), value(ch, py, px0 + 2), value(ch, py, px0 + 3));
    }
  }
}

// ------------------------------------------------------------------ fp32 linear (CUDA cores)
// 64 x 8 output tile per 128-thread block (each thread 1 row x 4 columns), K in chunks of 32
// streamed through a 3-stage cp.async ring so global latency overlaps the FMAs. Rows of x and w
// are read in 16-byte pieces (K, ldx, ldw multiples of 4; 16-byte aligned bases).
constexpr int LF_BM = 64, LF_BN = 8, LF_BK = 32, LF_ST = 3, LF_LD = LF_BK + 4, LF_THREADS = 128;

__device__ __forceinline__ void cp_async16_f(float* dst, const float* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(ok ? 16 : 0)
               : "memory");
}

__global__ void __launch_bounds__(LF_THREADS) linear_f32_kernel(const float* __restrict__ x, long long ldx,
                                                         const float* __restrict__ w, long long ldw,
                                                         const float* __restrict__ bias,
                                                         const float* __restrict__ bias2, float* __restrict__ y,
                                                         long long ldy, int M, int N, int K, int act) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ __align__(16) float xs[LF_ST][LF_BM][LF_LD];
  __shared__ __align__(16) float ws[LF_ST][LF_BN][LF_LD];
  const int m0 = blockIdx.y * LF_BM, n0 = blockIdx.x * LF_BN;
  const int tid = threadIdx.x;
  const int row = tid / 2, cg = (tid % 2) * 4;  // this thread: row m0 + row, columns n0 + cg .. +3
  const int nk = (K + LF_BK - 1) / LF_BK;

  auto load = [&](int kc, int st) {
    const int k0 = kc * LF_BK;
    // x: 64 rows x 8 chunks of 16 bytes, four per thread; w: 8 rows x 8 chunks
    for (int c = tid; c < LF_BM * (LF_BK / 4); c += LF_THREADS) {
      const int r = c / (LF_BK / 4), kk = (c % (LF_BK / 4)) * 4;
      const bool ok = m0 + r < M && k0 + kk < K;
      cp_async16_f(&xs[st][r][kk], x + (ok ? static_cast<long long>(m0 + r) * ldx + k0 + kk : 0), ok);
    }
    if (tid < LF_BN * (LF_BK / 4)) {
      const int r = tid / (LF_BK / 4), kk = (tid % (LF_BK / 4)) * 4;
      const bool ok = n0 + r < N && k0 + kk < K;
      cp_async16_f(&ws[st][r][kk], w + (ok ? static_cast<long long>(n0 + r) * ldw + k0 + kk : 0), ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  for (int st = 0; st < LF_ST - 1; ++st) {
    if (st < nk)
      load(st, st);
    else
      asm volatile("cp.async.commit_group;" ::: "memory");
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int kc = 0; kc < nk; ++kc) {
    const int nxt = kc + LF_ST - 1;
    if (nxt < nk)
      load(nxt, nxt % LF_ST);
    else
      asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(LF_ST - 1) : "memory");
    __syncthreads();
    const int st = kc % LF_ST;
#pragma unroll 8
    for (int kk = 0; kk < LF_BK; ++kk) {
      const float a = xs[st][row][kk];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(a, ws[st][cg + j][kk], acc[j]);
    }
    __syncthreads();
  }
  const int m = m0 + row;
  if (m < M) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + cg + j;
      if (n >= N) continue;
      float v = acc[j];
      if (bias) v += bias[n];
      if (bias2) v += bias2[n];
      if (act == 2) v = v / (1.0f + expf(-v));  // SiLU of the output, full fp32 accuracy
      y[static_cast<long long>(m) * ldy + n] = v;
    }
  }
}

// Many rows (the batched action / time MLP): 128 x 64 outputs per 256-thread CTA, each thread 8
// rows x 4 columns in registers. Both tiles sit k-major in shared memory (x is transposed as it is
// stored), so one k step is three 16-byte broadcast loads for 32 FMAs; the next k block's global
// loads are in registers during the current block's FMAs. Every output still accumulates over k in
// order with fmaf, so results equal linear_f32_kernel's bit for bit.
constexpr int LT_BM = 128, LT_BN = 64, LT_BK = 16, LT_THREADS = 256;

__global__ void __launch_bounds__(LT_THREADS) linear_f32_tiled_kernel(const float* __restrict__ x, long long ldx,
                                                                      const float* __restrict__ w, long long ldw,
                                                                      const float* __restrict__ bias,
                                                                      const float* __restrict__ bias2,
                                                                      float* __restrict__ y, long long ldy, int M,
                                                                      int N, int K, int act) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ __align__(16) float xs[2][LT_BK][LT_BM + 4];
  __shared__ __align__(16) float ws[2][LT_BK][LT_BN + 4];
  const int m0 = blockIdx.y * LT_BM, n0 = blockIdx.x * LT_BN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tr = (warp >> 1) * 4 + (lane >> 3);  // rows m0 + 8 tr .. +8
  const int tc = (warp & 1) * 8 + (lane & 7);    // columns n0 + 4 tc .. +4
  float4 rx[2], rw;
  auto gload = [&](int k0) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + i * LT_THREADS, r = c >> 2, k = k0 + (c & 3) * 4;
      rx[i] = (m0 + r < M && k < K) ? __ldg(reinterpret_cast<const float4*>(x + static_cast<long long>(m0 + r) * ldx + k))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int r = tid >> 2, k = k0 + (tid & 3) * 4;
    rw = (n0 + r < N && k < K) ? __ldg(reinterpret_cast<const float4*>(w + static_cast<long long>(n0 + r) * ldw + k))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  auto sstore = [&](int st) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + i * LT_THREADS, r = c >> 2, kq = (c & 3) * 4;
      xs[st][kq][r] = rx[i].x, xs[st][kq + 1][r] = rx[i].y, xs[st][kq + 2][r] = rx[i].z, xs[st][kq + 3][r] = rx[i].w;
    }
    const int r = tid >> 2, kq = (tid & 3) * 4;
    ws[st][kq][r] = rw.x, ws[st][kq + 1][r] = rw.y, ws[st][kq + 2][r] = rw.z, ws[st][kq + 3][r] = rw.w;
  };
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int nk = (K + LT_BK - 1) / LT_BK;
  gload(0);
  sstore(0);
  __syncthreads();
  for (int kc = 0; kc < nk; ++kc) {
    const int st = kc & 1;
    if (kc + 1 < nk) gload((kc + 1) * LT_BK);
#pragma unroll
    for (int kk = 0; kk < LT_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&xs[st][kk][tr * 8]);
      const float4 a1 = *reinterpret_cast<const float4*>(&xs[st][kk][tr * 8 + 4]);
      const float4 b = *reinterpret_cast<const float4*>(&ws[st][kk][tc * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (kc + 1 < nk) sstore(st ^ 1);  // that buffer was last read before the previous barrier
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + tr * 8 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tc * 4 + j;
      if (n >= N) continue;
      float v = acc[i][j];
      if (bias) v += bias[n];
      if (bias2) v += bias2[n];
      if (act == 2) v = v / (1.0f + expf(-v));  // SiLU of the output, full fp32 accuracy
      y[static_cast<long long>(m) * ldy + n] = v;
    }
  }
}

// ------------------------------------------------------------------ expert head + Euler step
// One block per row m: h = rms_norm(e[m]) in shared memory, then each warp computes output
// columns n = warp, warp + 8, ... as warp-reduced dot products; x_t[m, n] += dt * (h . w_n + b_n).
__global__ void expert_out_kernel(const float* __restrict__ e, long long lde, const float* __restrict__ norm_w,
                                  float eps, const float* __restrict__ w_out, const float* __restrict__ b_out,
                                  float* __restrict__ x_t, long long ldx, int N, int K, float dt) {
  grid_dep_launch();
  grid_dep_wait();
  extern __shared__ float h[];
  __shared__ float red[32];
  const long long m = blockIdx.x;
  const float* row = e + m * lde;
  float ss = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float v = row[k];
    h[k] = v;
    ss += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = rsqrtf(t / static_cast<float>(K) + eps);
  }
  __syncthreads();
  const float rstd = red[0];
  for (int k = threadIdx.x; k < K; k += blockDim.x) h[k] = (h[k] * rstd) * norm_w[k];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int n = warp; n < N; n += nw) {
    const float* wr = w_out + static_cast<long long>(n) * K;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) acc = fmaf(h[k], wr[k], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) x_t[m * ldx + n] += dt * (acc + b_out[n]);
  }
}

// ------------------------------------------------------------------ prefix tail rows
// grid (observations, chunks of 256 tail elements): element (r, c) of the (lang_len + 1) x d tail
// is the task-token row r copied, or for r == lang_len the state row
// state_w @ pad((state - mean) / (std + 1e-8)) + state_b.
__global__ void prefix_tail_kernel(const float* __restrict__ state, int state_dim, const float* __restrict__ s_mean,
                                   const float* __restrict__ s_std, const float* __restrict__ state_w, int max_state,
                                   const float* __restrict__ state_b, const float* __restrict__ lang, int lang_len,
                                   int d, float* __restrict__ prefix, long long ldp, long long prefix_rows,
                                   long long tail_row) {
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x;
  const long long idx = static_cast<long long>(blockIdx.y) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(lang_len + 1) * d) return;
  const int r = static_cast<int>(idx / d), c = static_cast<int>(idx % d);
  float* dst = prefix + (static_cast<long long>(b) * prefix_rows + tail_row + r) * ldp + c;
  if (r < lang_len) {
    *dst = lang[static_cast<long long>(r) * d + c];
    return;
  }
  float acc = 0.f;
  for (int j = 0; j < state_dim; ++j) {
    const float st = (state[static_cast<long long>(b) * state_dim + j] - s_mean[j]) / (s_std[j] + 1e-8f);
    acc = fmaf(st, state_w[static_cast<long long>(c) * max_state + j], acc);
  }
  *dst = acc + state_b[c];
}

// ------------------------------------------------------------------ unnormalisation
__global__ void finish_kernel(const float* __restrict__ x_t, int max_action, const float* __restrict__ state,
                              int state_dim, const float* __restrict__ s_mean, const float* __restrict__ s_std,
                              const float* __restrict__ r_mean, const float* __restrict__ r_std,
                              const float* __restrict__ a_mean, const float* __restrict__ a_std,
                              float* __restrict__ out, int action_dim, int H, int repr) {
  grid_dep_launch();
  grid_dep_wait();
  const int b = blockIdx.x, col = threadIdx.x;
  if (col >= action_dim) return;
  const float* x = x_t + static_cast<long long>(b) * H * max_action;
  float st = 0.f;
  if (repr != 0 && col < state_dim) st = (state[b * state_dim + col] - s_mean[col]) / (s_std[col] + 1e-8f);
  float run = 0.f;
  for (int i = 0; i < H; ++i) {
    float a = x[i * max_action + col];
    if (repr != 0) {
      a = a * r_std[col] + r_mean[col];
      if (repr == 1) {
        a = a + st;
      } else {
        run += a;
        a = st + run;
      }
    }
    out[(static_cast<long long>(b) * H + i) * action_dim + col] = a * a_std[col] + a_mean[col];
  }
}

// Preprocessed frames px (n, 3, S, S) float -> patch rows (n * G^2, 3 P^2): one thread per patch
// row segment (image, patch, channel, row py): P consecutive floats of px in, P values out.
__global__ void patchify_kernel(const float* __restrict__ px, int n_img, int S, int P, void* __restrict__ out,
                                int y_type, float qs) {
  grid_dep_launch();
  grid_dep_wait();
  const int G = S / P;
  const long long segs = static_cast<long long>(n_img) * G * G * 3 * P;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= segs) return;
  const int py = static_cast<int>(i % P);
  const int c = static_cast<int>((i / P) % 3);
  const long long row = i / (3 * P);  // patch row: image * G^2 + gy * G + gx
  const int im = static_cast<int>(row / (G * G)), pr = static_cast<int>(row % (G * G));
  const int gy = pr / G, gx = pr % G;
  const float* src = px + ((static_cast<long long>(im) * 3 + c) * S + gy * P + py) * S + gx * P;
  const long long o = row * 3 * P * P + (c * P + py) * P;
  for (int x = 0; x < P; ++x) {
    const float v = src[x];
    if (y_type == SO101_BF16)
      static_cast<__nv_bfloat16*>(out)[o + x] = __float2bfloat16_rn(v);
    else if (y_type == SO101_I8)
      static_cast<int8_t*>(out)[o + x] = quant_i8(v, qs);
    else
      static_cast<float*>(out)[o + x] = v;
  }
}

// x (M x K fp32) -> y (M x 3K bf16) = [hi | hi | lo] with hi = bf16(x), lo = bf16(x - hi): the
// operand of a bf16 GEMM against [W_hi | W_lo | W_hi] that sums x_hi W_hi + x_hi W_lo + x_lo W_hi
// (the two-term split of each operand, its lo x lo product dropped): an fp32 linear on the tensor
// cores to about 2^-16 relative. One thread per 4 columns.
__global__ void split_bf16x3_kernel(const float* __restrict__ x, long long ldx, int M, int K,
                                    __nv_bfloat16* __restrict__ y, long long ldy) {
  grid_dep_launch();
  grid_dep_wait();
  const int q4 = K / 4;
  const long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (i >= static_cast<long long>(M) * q4) return;
  const long long m = i / q4;
  const int c = static_cast<int>(i % q4) * 4;
  const float4 v = *reinterpret_cast<const float4*>(x + m * ldx + c);
  const __nv_bfloat162 h01 = __floats2bfloat162_rn(v.x, v.y), h23 = __floats2bfloat162_rn(v.z, v.w);
  const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
  const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - f01.x, v.y - f01.y);
  const __nv_bfloat162 l23 = __floats2bfloat162_rn(v.z - f23.x, v.w - f23.y);
  uint2 hi, lo;
  hi.x = *reinterpret_cast<const uint32_t*>(&h01), hi.y = *reinterpret_cast<const uint32_t*>(&h23);
  lo.x = *reinterpret_cast<const uint32_t*>(&l01), lo.y = *reinterpret_cast<const uint32_t*>(&l23);
  __nv_bfloat16* row = y + m * ldy + c;
  *reinterpret_cast<uint2*>(row) = hi;
  *reinterpret_cast<uint2*>(row + K) = hi;
  *reinterpret_cast<uint2*>(row + 2 * K) = lo;
}

}  // namespace so101

using namespace so101;

extern "C" int so101_split_bf16x3(const float* x, int64_t ldx, int64_t M, int64_t K, void* y, int64_t ldy,
                                  cudaStream_t stream) {
  if (!x || !y || M <= 0 || K <= 0 || K % 4 || ldx < K || ldx % 4 || ldy < 3 * K || ldy % 4) return SO101_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 8 || M > 0x7fffffffLL || K > (1 << 24))
    return SO101_ERR_ARG;
  const long long blocks = (M * (K / 4) + 255) / 256;
  if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(split_bf16x3_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, x, ldx,
                       static_cast<int>(M), static_cast<int>(K), static_cast<__nv_bfloat16*>(y), ldy);
}

extern "C" int so101_patchify(const float* px, int n_img, int S, int P, void* patches, int y_type, float y_qscale,
                              cudaStream_t stream) {
  if (!px || !patches || n_img <= 0 || P <= 0 || S <= 0 || S % P) return SO101_ERR_ARG;
  if (y_type != SO101_BF16 && y_type != SO101_I8 && y_type != SO101_F32) return SO101_ERR_ARG;
  if (y_type == SO101_I8 && !(y_qscale > 0.f)) return SO101_ERR_ARG;
  const long long G = S / P;
  const long long segs = static_cast<long long>(n_img) * G * G * 3 * P;
  const long long blocks = (segs + 255) / 256;
  if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(patchify_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, px, n_img,
                       static_cast<int>(S), static_cast<int>(P), patches, y_type, y_qscale);
}

extern "C" int so101_preprocess(const uint8_t* img, int n_img, int h, int w, int rh, int rw, int S, int P,
                                void* patches, int y_type, float y_qscale, cudaStream_t stream) {
  if (!img || !patches || n_img <= 0 || h <= 0 || w <= 0 || P <= 0 || S % P) return SO101_ERR_ARG;
  if (rh <= 0 || rw <= 0 || rh > S || rw > S || (3 * P * P) % 2) return SO101_ERR_ARG;
  if (y_type == SO101_I8 && !(y_qscale > 0.f)) return SO101_ERR_ARG;
  const long long G = S / P;
  if (h == S && w == S && rh == S && rw == S && P == 16 && (S * 3) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(img) % 16 == 0 && reinterpret_cast<uintptr_t>(patches) % 16 == 0) {
    const long long blocks = (n_img * G * G + kPpWarps - 1) / kPpWarps;
    if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
    return launch_kernel(preprocess_patch_kernel, dim3(static_cast<unsigned>(blocks)), dim3(32 * kPpWarps), 0, stream,
                         img, n_img, S, patches, y_type, y_qscale);
  }
  const long long pairs = n_img * G * G * (3 * P * P / 2);
  const long long blocks = (pairs + 255) / 256;
  if (blocks > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(preprocess_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream,
                       img, n_img, h, w, rh, rw, S, P, patches,
                                                                        y_type, y_qscale);
}

extern "C" int so101_linear_f32(const float* x, int64_t ldx, const float* w, int64_t ldw, const float* bias,
                                const float* bias2, float* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                                int act, cudaStream_t stream) {
  if (!x || !w || !y || M <= 0 || N <= 0 || K <= 0 || ldx < K || ldw < K || ldy < N) return SO101_ERR_ARG;
  if (K % 4 || ldx % 4 || ldw % 4 || reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16)
    return SO101_ERR_ARG;
  if (M >= 512) {  // enough rows for register-blocked 128 x 64 tiles
    const long long ty = (M + LT_BM - 1) / LT_BM, tx = (N + LT_BN - 1) / LT_BN;
    if (ty > 65535 || tx > 0x7fffffffLL) return SO101_ERR_ARG;
    return launch_kernel(linear_f32_tiled_kernel, dim3(static_cast<unsigned>(tx), static_cast<unsigned>(ty)),
                         dim3(LT_THREADS), 0, stream, x, ldx, w, ldw, bias, bias2, y, ldy, static_cast<int>(M),
                         static_cast<int>(N), static_cast<int>(K), act);
  }
  const long long gy = (M + LF_BM - 1) / LF_BM, gx = (N + LF_BN - 1) / LF_BN;
  if (gy > 65535 || gx > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(linear_f32_kernel, dim3(dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy))), dim3(LF_THREADS), 0, stream,
                       x, ldx, w, ldw, bias, bias2, y, ldy, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), act);
}

extern "C" int so101_expert_out(const float* e, int64_t lde, const float* norm_w, float eps, const float* w_out,
                                const float* b_out, float* x_t, int64_t ldx, int64_t M, int64_t N, int64_t K,
                                float dt, cudaStream_t stream) {
  if (!e || !norm_w || !w_out || !b_out || !x_t || M <= 0 || N <= 0 || K <= 0 || K > 8192) return SO101_ERR_ARG;
  if (M > 0x7fffffffLL) return SO101_ERR_ARG;
  return launch_kernel(expert_out_kernel, dim3(static_cast<unsigned>(M)), dim3(256), K * sizeof(float), stream,
                       e, lde, norm_w, eps, w_out, b_out, x_t, ldx, static_cast<int>(N), static_cast<int>(K), dt);
}

extern "C" int so101_prefix_tail(const float* state, int state_dim, const float* s_mean, const float* s_std,
                                 const float* state_w, int max_state, const float* state_b, const float* lang,
                                 int lang_len, int d, float* prefix, int64_t ldp, int64_t prefix_rows,
                                 int64_t tail_row, int batch, cudaStream_t stream) {
  if (!state || !s_mean || !s_std || !state_w || !state_b || !prefix || batch <= 0 || d <= 0) return SO101_ERR_ARG;
  if (lang_len > 0 && !lang) return SO101_ERR_ARG;
  if (state_dim > max_state || max_state <= 0 || max_state > 4096) return SO101_ERR_ARG;
  const long long chunks = (static_cast<long long>(lang_len + 1) * d + 255) / 256;
  if (chunks > 65535) return SO101_ERR_ARG;
  return launch_kernel(prefix_tail_kernel, dim3(batch, static_cast<unsigned>(chunks)), dim3(256), 0, stream, state, state_dim, s_mean, s_std, state_w,
                                                                         max_state, state_b, lang, lang_len, d,
                                                                         prefix, ldp, prefix_rows, tail_row);
}

extern "C" int so101_finish(const float* x_t, int max_action, const float* state, int state_dim,
                            const float* s_mean, const float* s_std, const float* r_mean, const float* r_std,
                            const float* a_mean, const float* a_std, float* out, int action_dim, int H, int repr,
                            int batch, cudaStream_t stream) {
  if (!x_t || !state || !s_mean || !s_std || !r_mean || !r_std || !a_mean || !a_std || !out) return SO101_ERR_ARG;
  if (batch <= 0 || H <= 0 || action_dim <= 0 || action_dim > max_action || action_dim > 1024) return SO101_ERR_ARG;
  if (repr < 0 || repr > 2) return SO101_ERR_ARG;
  return launch_kernel(finish_kernel, dim3(batch), dim3(((action_dim + 31) / 32) * 32), 0, stream, x_t, max_action, state, state_dim, s_mean,
                                                                       s_std, r_mean, r_std, a_mean, a_std, out,
                                                                       action_dim, H, repr);
}
