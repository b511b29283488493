// SigLIP patch embedding straight from the camera frames: the reference's preprocessing
// (uint8 -> /255 -> *2-1, Engine._vision at pkg/model/engine.py:236-245, identity resize at S x S)
// and patch unfold (pkg/model/smolvla.py:166-168) folded into the A-operand producer of the patch
// GEMM, so the patch rows never exist in global memory:
//   y[m, n] = sum_k A[m, k] W[n, k] + bias[n] + pos[m % period, n],
//   A[m, k] = bf16(img[im][16 gy + py][16 gx + px][c] / 255 * 2 - 1),  k = 256 c + 16 py + px,
// with m = im * G^2 + gy * G + gx the patch row (G = S / 16).
//
// Persistent, one CTA per SM. A CTA takes 128-patch row blocks in turn; 128 consecutive patches are
// 128 / G whole patch rows of one frame, so their pixels are one contiguous run of 128 * 768 bytes,
// brought into shared memory by bulk copies once per row block. For each 256-feature output tile
// of the block (an item) the K = 768 reduction runs as twelve 64-wide blocks through a two-stage
// ring, into one of two TMEM accumulators, so the epilogue of item i overlaps the main loop of i+1:
//   warp 0 (one thread)  bulk copies of the pixel run; TMA of the weight blocks (256 x 64, SW128)
//   warp 1 (one thread)  tcgen05.mma M = 128, N = 256, K = 16 x 4 per block
//   warps 2-5            A producer: thread r converts its patch's 4 x 16 pixels of one channel per
//                        K block from the staged run (three 16-byte loads per pixel row) through a
//                        256-entry bf16 table of (v / 255) * 2 - 1 into the swizzled K-major tile
//   warps 6-13           epilogue: TMEM -> + bias + position row -> fp32 rows (two threads a row)
// The K blocks go in the plain order 0..11 with the values the standalone preprocessing writes, so
// the accumulators are bit-identical to so101_preprocess followed by so101_gemm without a K split.
#include "common.cuh"

namespace so101 {

struct PatchArgs {
  const uint8_t* img;  // (n_img, S, S, 3)
  int S, G;            // frame side, patches per side
  long long M;         // n_img * G^2 patch rows
  int N;               // output features (multiple of 256)
  int m_tiles;         // 128-patch row blocks
  const float* bias;   // N, or null
  const float* pos;    // (period, N) added per row m % period, or null
  long long period;
  float* y;
  long long ldy;
  int* status;
};

constexpr int kPeThreads = 448;        // warps 0-1 copies / MMA, 2-5 A producer, 6-13 epilogue
constexpr int kPeStages = 2;
constexpr int kPeABlk = 128 * 128;     // 128 rows x 64 bf16
constexpr int kPeBBlk = 256 * 128;     // 256 rows x 64 bf16
constexpr int kPeStage = kPeABlk + kPeBBlk;
constexpr int kPeKb = 12;              // 768 / 64
constexpr int kPeRaw = 128 * 768;      // one row block's pixels
constexpr int kPeOffRaw = kPeStages * kPeStage;
constexpr int kPeOffBar = kPeOffRaw + kPeRaw;
constexpr int kPeOffLut = kPeOffBar + 256;
constexpr int kPeSmem = kPeOffLut + 512 + 1024;
static_assert(kPeSmem <= 232448, "227 KB of shared memory per CTA");

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// One channel of a 16-pixel run (48 interleaved RGB bytes in three 16-byte words) as 16 bf16
// values packed in pairs, through the conversion table; compile-time byte positions keep the run in
// registers.
template <int C>
__device__ __forceinline__ void pe_channel(const uint4 (&u)[3], const __nv_bfloat16* lut, bool live,
                                           uint32_t (&w)[8]) {
  const uint32_t words[12] = {u[0].x, u[0].y, u[0].z, u[0].w, u[1].x, u[1].y,
                              u[1].z, u[1].w, u[2].x, u[2].y, u[2].z, u[2].w};
#pragma unroll
  for (int px = 0; px < 16; px += 2) {
    const int j0 = px * 3 + C, j1 = (px + 1) * 3 + C;
    const uint32_t v0 = (words[j0 >> 2] >> ((j0 & 3) * 8)) & 0xFFu;
    const uint32_t v1 = (words[j1 >> 2] >> ((j1 & 3) * 8)) & 0xFFu;
    const uint32_t lo = live ? __bfloat16_as_ushort(lut[v0]) : 0u;
    const uint32_t hi = live ? __bfloat16_as_ushort(lut[v1]) : 0u;
    w[px >> 1] = lo | (hi << 16);
  }
}

__global__ void __launch_bounds__(kPeThreads, 1) patch_embed_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                   const PatchArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + kPeOffBar);  // [2] 4 producer warps
  uint64_t* b_full = a_full + kPeStages;                               // [2] TMA bytes
  uint64_t* empty = b_full + kPeStages;                                // [2] MMA commit
  uint64_t* acc_full = empty + kPeStages;                              // [2] MMA commit
  uint64_t* acc_empty = acc_full + 2;                                  // [2] 8 epilogue warps
  uint64_t* raw_full = acc_empty + 2;                                  // bulk-copy bytes
  uint64_t* raw_free = raw_full + 1;                                   // 4 producer warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(raw_free + 1);
  __nv_bfloat16* lut = reinterpret_cast<__nv_bfloat16*>(smem + kPeOffLut);
  uint8_t* raw = smem + kPeOffRaw;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int n_nt = a.N / 256;
  // this CTA's items: row blocks blockIdx.x, blockIdx.x + gridDim.x, ..., each with n_nt tiles
  const int my_blocks = a.m_tiles > static_cast<int>(blockIdx.x)
                            ? (a.m_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                                  static_cast<int>(gridDim.x)
                            : 0;
  const int items = my_blocks * n_nt;

  if (t == 0) {
    for (int s = 0; s < kPeStages; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&b_full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    mbar_init(raw_full, 1);
    mbar_init(raw_free, 4);
    fence_mbar_init();
  }
  for (int v = t; v < 256; v += kPeThreads) {
    const float x = static_cast<float>(v) / 255.0f;  // the preprocessing's own arithmetic
    lut[v] = __float2bfloat16_rn(x * 2.0f - 1.0f);
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
      tma_prefetch_desc(&tm_w);
      const uint64_t pol = policy_evict_last();
      int kb = 0;  // K blocks issued so far (ring position)
      bool ok = true;
      for (int it = 0; it < items && ok; ++it) {
        const int blk = it / n_nt, nt = it % n_nt;
        if (nt == 0) {
          // the row block's pixels, once the producers are done with the previous block's
          if (blk > 0 && !mbar_wait(raw_free, static_cast<uint32_t>(blk - 1) & 1u, a.status)) {
            ok = false;
            break;
          }
          if (blk == 0) grid_dep_wait();  // the frames may come from the previous grid
          const long long mt = blockIdx.x + static_cast<long long>(blk) * gridDim.x;
          const uint8_t* src = a.img + mt * static_cast<long long>(kPeRaw);
          const long long left = a.M * 768 - mt * static_cast<long long>(kPeRaw);
          const uint32_t bytes = static_cast<uint32_t>(left < kPeRaw ? left : kPeRaw);
          mbar_arrive_expect_tx(raw_full, bytes);
          for (uint32_t off = 0; off < bytes; off += 16384)
            bulk_load(raw + off, src + off, bytes - off < 16384 ? bytes - off : 16384, raw_full);
        }
        for (int i = 0; i < kPeKb; ++i, ++kb) {
          const int s = kb % kPeStages;
          if (kb >= kPeStages && !mbar_wait(&empty[s], static_cast<uint32_t>(kb / kPeStages - 1) & 1u, a.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[s], kPeBBlk);
          tma_load_2d(smem + s * kPeStage + kPeABlk, &tm_w, &b_full[s], i * 64, nt * 256, pol);
        }
      }
      // every copy lands before the CTA may leave (only an unwinding run has any left in flight)
      for (int j = kb > kPeStages ? kb - kPeStages : 0; j < kb; ++j)
        mbar_wait(&b_full[j % kPeStages], static_cast<uint32_t>(j / kPeStages) & 1u, a.status);
      if (items > 0) mbar_wait(raw_full, static_cast<uint32_t>(my_blocks - 1) & 1u, a.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_bf16(128, 256);
      int kb = 0;
      bool ok = true;
      for (int it = 0; it < items && ok; ++it) {
        const int buf = it & 1;
        // the epilogue has drained this accumulator's previous item
        if (it >= 2 && !mbar_wait(&acc_empty[buf], static_cast<uint32_t>(it / 2 - 1) & 1u, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int i = 0; i < kPeKb; ++i, ++kb) {
          const int s = kb % kPeStages;
          const uint32_t ph = static_cast<uint32_t>(kb / kPeStages) & 1u;
          ok = mbar_wait(&a_full[s], ph, a.status) && mbar_wait(&b_full[s], ph, a.status);
          if (!ok) break;
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * kPeStage);
          const uint64_t ad = sw128_desc(base), bd = sw128_desc(base + kPeABlk);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16(tmem + buf * 256, ad + 2 * k, bd + 2 * k, kIdesc, (i > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (ok)
          mma_commit(&acc_full[buf]);
        else
          mbar_arrive(&acc_full[buf]);  // unwind: the epilogue finds the error recorded
      }
    }
  } else if (warp < 6) {
    // ---------------- A producer: thread r = row r of each 128-patch block
    const int r = t - 64;
    int kb = 0;
    bool ok = true;
    for (int it = 0; it < items && ok; ++it) {
      const int blk = it / n_nt, nt = it % n_nt;
      const long long mt = blockIdx.x + static_cast<long long>(blk) * gridDim.x;
      const long long m = mt * 128 + r;
      const bool live = m < a.M;
      if (nt == 0 && !mbar_wait(raw_full, static_cast<uint32_t>(blk) & 1u, a.status)) {
        ok = false;
        break;
      }
      // patch m in the staged run: patch row (m / G) % (128 / G) of the block, column m % G
      const int gyl = (r / a.G), gx = r % a.G;
      const uint8_t* src = raw + static_cast<long long>(gyl) * 16 * a.S * 3 + gx * 48;
      for (int i = 0; i < kPeKb; ++i, ++kb) {
        const int s = kb % kPeStages;
        if (kb >= kPeStages && !mbar_wait(&empty[s], static_cast<uint32_t>(kb / kPeStages - 1) & 1u, a.status)) {
          ok = false;
          break;
        }
        const int c = i >> 2, py0 = (i & 3) * 4;  // K block i: channel c, patch rows py0..py0+3
        uint8_t* arow = smem + s * kPeStage + r * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4* run = reinterpret_cast<const uint4*>(src + (py0 + q) * a.S * 3);
          uint4 u[3];
          u[0] = run[0];
          u[1] = run[1];
          u[2] = run[2];
          uint32_t w[8];
          if (c == 0)
            pe_channel<0>(u, lut, live, w);
          else if (c == 1)
            pe_channel<1>(u, lut, live, w);
          else
            pe_channel<2>(u, lut, live, w);
          // K elements 16 q .. 16 q + 15 of this block: 16-byte chunks 2 q and 2 q + 1 of the row
          *reinterpret_cast<uint4*>(arow + (((2 * q) ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(arow + (((2 * q + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
      if (nt == n_nt - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(raw_free);  // the pixel run may be overwritten
      }
    }
  } else {
    // ---------------- epilogue (8 warps): thread = TMEM lane = tile row, one 128-column half each;
    // a 32-column chunk's accumulators, biases and position values are all loaded before any use
    grid_dep_wait();  // y may still be read by the previous grid
    const int wq = warp & 3, row = wq * 32 + lane, half = (warp - 6) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(wq * 32) << 16);
    for (int it = 0; it < items; ++it) {
      const int buf = it & 1, blk = it / n_nt, nt = it % n_nt;
      const long long m = (blockIdx.x + static_cast<long long>(blk) * gridDim.x) * 128 + row;
      const float* prow = a.pos ? a.pos + (m % a.period) * a.N : nullptr;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], static_cast<uint32_t>(it / 2) & 1u,
                                                        a.status) ? 1 : 0) != 0;
      tc_fence_after();
      const bool live = ok && m < a.M;
#pragma unroll 1
      for (int c = half * 128; c < half * 128 + 128; c += 32) {
        uint32_t v[2][16];
        tmem_ld16(lane_addr + buf * 256 + c, v[0]);
        tmem_ld16(lane_addr + buf * 256 + c + 16, v[1]);
        const int n = nt * 256 + c;
        float4 bv[8], pv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          bv[j] = a.bias ? __ldg(reinterpret_cast<const float4*>(a.bias + n) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
          pv[j] = prow ? __ldg(reinterpret_cast<const float4*>(prow + n) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        tmem_ld_wait();
        if (live) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t* r = v[j >> 2] + 4 * (j & 3);
            float4 x = make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]), __uint_as_float(r[2]),
                                   __uint_as_float(r[3]));
            // (acc + bias) + position, in that order, as the GEMM's residual epilogue adds them
            if (a.bias) x.x += bv[j].x, x.y += bv[j].y, x.z += bv[j].z, x.w += bv[j].w;
            if (prow) x.x += pv[j].x, x.y += pv[j].y, x.z += pv[j].z, x.w += pv[j].w;
            *reinterpret_cast<float4*>(a.y + m * a.ldy + n + 4 * j) = x;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

namespace {

using PeEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PeEncodeFn pe_encode() {
  static PeEncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PeEncodeFn>(p);
    return static_cast<PeEncodeFn>(nullptr);
  }();
  return fn;
}

}  // namespace

}  // namespace so101

using namespace so101;

extern "C" int so101_patch_embed(const uint8_t* img, int n_img, int S, const void* w, int64_t ldw, int64_t N,
                                 const float* bias, const float* pos, int64_t period, float* y, int64_t ldy,
                                 cudaStream_t stream) {
  if (!img || !w || !y || n_img <= 0 || S <= 0 || S % 16 || N <= 0 || N % 256 || N > (1 << 20)) return SO101_ERR_ARG;
  if (ldw < 768 || (ldw * 2) % 16 || ldy < N || ldy % 4 || (pos && period <= 0)) return SO101_ERR_ARG;
  const auto al16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (!al16(img) || !al16(w) || !al16(y) || (bias && !al16(bias)) || (pos && !al16(pos))) return SO101_ERR_ARG;
  const long long G = S / 16;
  // 128 consecutive patches must be whole patch rows of one frame (one contiguous pixel run)
  if (128 % G || (G * G) % 128) return SO101_ERR_ARG;
  const long long M = static_cast<long long>(n_img) * G * G;
  const long long tiles_m = (M + 127) / 128;
  if (tiles_m > 0x7fffffffLL || N / 256 > 65535) return SO101_ERR_ARG;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  PeEncodeFn enc = pe_encode();
  if (!enc) return SO101_ERR_DRIVER;
  CUtensorMap tm;
  cuuint64_t dims[2] = {768, static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw) * 2};
  cuuint32_t box[2] = {64, 256};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return SO101_ERR_ARG;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(patch_embed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeSmem);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  PatchArgs a;
  a.img = img;
  a.S = S;
  a.G = static_cast<int>(G);
  a.M = M;
  a.N = static_cast<int>(N);
  a.m_tiles = static_cast<int>(tiles_m);
  a.bias = bias;
  a.pos = pos;
  a.period = pos ? period : 1;
  a.y = y;
  a.ldy = ldy;
  a.status = status_ptr();
  const long long grid = tiles_m < sms ? tiles_m : sms;
  return launch_kernel(patch_embed_kernel, dim3(static_cast<unsigned>(grid)), dim3(kPeThreads), kPeSmem, stream, tm,
                       a);
}
