// The SwiGLU MLP block of the action expert at batch 1 in one launch:
//   y = residual + (silu(rs * x W_gate^T) * (rs * x W_up^T)) W_down^T
// with x = bf16(e * ln_post) (the residual stream times the norm weight, written by the previous
// epilogue) and rs the row's RMSNorm scale from its statistics slots, so the norm is finished here
// as in the GEMMs. One launch instead of a gate/up GEMM launch followed by a down GEMM launch.
//
// The down projection's K dimension is the MLP's hidden features, so a cluster of S = mlp / 128
// CTAs shares it: CTA r (cluster rank) owns hidden features [128 r, 128 r + 128). There is one
// cluster per 128-feature output tile (and observation). Each CTA
//   1  loads its W_down block (128 outputs x 128 hidden, two SWIZZLE_128B boxes) and the first
//      stages of its gate and up rows before waiting for the previous grid (weights are constant);
//   2  streams K in 64-wide blocks: gate rows, up rows and the token rows x through a TMA ring,
//      two M=128, N=64 tcgen05.mma per 16-wide K step into two TMEM accumulators (gate, up);
//   3  applies the token's RMSNorm scale and silu(gate) * up in fp32 and writes the bf16 hidden
//      activations straight into a shared-memory K-major tile, the B operand of the down MMA;
//   4  multiplies its W_down block by that tile (K = 128): its partial of the output tile, staged
//      to shared memory;
//   5  after a cluster barrier, sums whole tokens over the S partials through DSMEM in rank order
//      (deterministic) and runs the residual epilogue (token_reduce.cuh).
// Every output tile's cluster recomputes all hidden activations: the gate/up weights are read once
// per output tile, from L2 after the first; in exchange no hidden activation crosses global memory
// and the down GEMM's dependent launch disappears. Every wait is bounded (SO101_ERR_TIMEOUT).
#include <mutex>

#include "token_reduce.cuh"

namespace so101 {

constexpr int kMlpThreads = 512;  // four threads per TMEM lane in the epilogues
constexpr int kMlpMaxCluster = 16;
constexpr int kMlpStages = 3;  // 4 stages and L2 prefetches of the later blocks measured no faster
constexpr int kMlpWBlk = 128 * 128;                      // 128 rows x 64 bf16
constexpr int kMlpXBlk = 64 * 128;                       // 64 rows x 64 bf16
constexpr int kMlpStage = 2 * kMlpWBlk + kMlpXBlk;       // gate, up, x: 40 KB
constexpr int kMlpOffDown = kMlpStages * kMlpStage;      // W_down block, two K halves: 32 KB
constexpr int kMlpOffAct = kMlpOffDown + 2 * kMlpWBlk;   // hidden activations, two K halves: 16 KB
constexpr int kMlpOffBar = kMlpOffAct + 2 * kMlpXBlk;    // barriers, TMEM slot, token scales
constexpr int kMlpSmem = kMlpOffBar + 128 + 64 * 4 + 1024;
static_assert(kMlpStages * kMlpStage >= 64 * 128 * 4, "the fp32 partial reuses the ring");

struct MlpArgs {
  TokenEpilogue ep;
  int rows;  // token rows per observation (<= 64)
  int kb;    // 64-wide K blocks of the input
  int mlp;   // hidden features (gate rows; up rows follow)
  const float* rms_ss;
  int rms_slots;
  long long rms_ld;
  float rms_n, rms_eps;
  int* status;
};

__device__ __forceinline__ void mlp_fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// The row's RMSNorm scale from its statistics slots, summed in slot order (as the GEMMs do).
__device__ __forceinline__ float mlp_rms_scale(const MlpArgs& a, long long row) {
  const float* r = a.rms_ss + row * a.rms_ld;
  float s = 0.f;
  for (int i = 0; i < a.rms_slots; ++i) s += r[i];
  return rsqrtf(s / a.rms_n + a.rms_eps);
}

__global__ void __launch_bounds__(kMlpThreads, 1) mlp_kernel(const __grid_constant__ CUtensorMap tm_x,
                                                          const __grid_constant__ CUtensorMap tm_gu,
                                                          const __grid_constant__ CUtensorMap tm_down,
                                                          const MlpArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kMlpOffBar);
  uint64_t* empty = full + kMlpStages;
  uint64_t* accum = empty + kMlpStages;
  uint64_t* down_full = accum + 1;
  uint64_t* down_done = down_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(down_done + 1);
  float* rtab = reinterpret_cast<float*>(smem + kMlpOffBar + 128);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int r = blockIdx.x, tile = blockIdx.y, bi = blockIdx.z;
  const long long row0 = static_cast<long long>(bi) * a.rows;
  constexpr uint32_t kCols = 256;  // gate [0, 64), up [64, 128), down [128, 192)
  constexpr uint32_t kIdesc = idesc_bf16(128, 64);

  if (t == 0) {
    for (int s = 0; s < kMlpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    mbar_init(down_full, 1);
    mbar_init(down_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dep_launch();

  if (warp == 0 && lane == 0) {
    // TMA producer: W_down and the first stages' gate/up rows go out before the previous grid ends
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_gu);
    tma_prefetch_desc(&tm_down);
    const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
    mbar_arrive_expect_tx(down_full, 2 * kMlpWBlk);
    tma_load_2d(smem + kMlpOffDown, &tm_down, down_full, r * 128, tile * 128, pol_w);
    tma_load_2d(smem + kMlpOffDown + kMlpWBlk, &tm_down, down_full, r * 128 + 64, tile * 128, pol_w);
    // the ring's first round of gate/up rows, then (once the previous grid is done) its tokens
    const int pre = min(kMlpStages, a.kb);
    for (int i = 0; i < pre; ++i) {
      uint8_t* st = smem + i * kMlpStage;
      mbar_arrive_expect_tx(&full[i], kMlpStage);
      tma_load_2d(st, &tm_gu, &full[i], i * 64, r * 128, pol_w);
      tma_load_2d(st + kMlpWBlk, &tm_gu, &full[i], i * 64, a.mlp + r * 128, pol_w);
    }
    grid_dep_wait();
    for (int i = 0; i < pre; ++i)
      tma_load_2d(smem + i * kMlpStage + 2 * kMlpWBlk, &tm_x, &full[i], i * 64, static_cast<int>(row0), pol_x);
    for (int i = pre; i < a.kb; ++i) {
      const int s = i % kMlpStages;
      const uint32_t round = static_cast<uint32_t>(i / kMlpStages);
      if (!mbar_wait(&empty[s], (round - 1) & 1u, a.status)) break;
      uint8_t* st = smem + s * kMlpStage;
      mbar_arrive_expect_tx(&full[s], kMlpStage);
      tma_load_2d(st, &tm_gu, &full[s], i * 64, r * 128, pol_w);
      tma_load_2d(st + kMlpWBlk, &tm_gu, &full[s], i * 64, a.mlp + r * 128, pol_w);
      tma_load_2d(st + 2 * kMlpWBlk, &tm_x, &full[s], i * 64, static_cast<int>(row0), pol_x);
    }
  } else if (warp == 1) {
    // MMA issuer, gate and up accumulators: the whole warp runs the waits (outcomes made
    // warp-uniform), its elected lane issues and commits
    bool ok = true;
    for (int i = 0; i < a.kb && ok; ++i) {
      const int s = i % kMlpStages;
      const uint32_t round = static_cast<uint32_t>(i / kMlpStages);
      ok = __all_sync(0xffffffffu, mbar_wait(&full[s], round & 1u, a.status));
      if (!ok) break;
      tc_fence_after();
      const uint32_t base = smem_u32(smem + s * kMlpStage);
      const uint64_t ag = sw128_desc(base), au = sw128_desc(base + kMlpWBlk), bx = sw128_desc(base + 2 * kMlpWBlk);
      if (elect_one()) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
          mma_f16(tmem, ag + 2 * k, bx + 2 * k, kIdesc, acc);
          mma_f16(tmem + 64, au + 2 * k, bx + 2 * k, kIdesc, acc);
        }
        mma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (elect_one()) {
      if (ok)
        mma_commit(accum);
      else
        mbar_arrive(accum);  // a stage never came: unwind with the error recorded
    }
    grid_dep_wait();
  } else {
    grid_dep_wait();
    if (warp >= 2) {
      // the tokens' RMSNorm scales while the MMAs run (the statistics are complete once the
      // previous grid is)
      for (int i = t - 64; i < 64; i += 64)
        rtab[i] = (a.rms_ss && i < a.rows) ? mlp_rms_scale(a, row0 + i) : 1.f;
    }
  }
  __syncwarp();
  __syncthreads();  // rtab

  const int nv = a.rows;
  const TokenPrefetch pf = token_prefetch<kMlpThreads>(a.ep, static_cast<int>(gridDim.x), nv, row0, tile);
  // thread t reads TMEM lane tl (warp w: lanes 32 (w % 4) ..) and the 16-token chunks of parity hh
  const int tl = t & 127, hh = t >> 7;
  const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  const bool acc_ok = __all_sync(0xffffffffu, mbar_wait(accum, 0, a.status) ? 1 : 0) != 0;
  tc_fence_after();
  // hidden feature tl of this CTA's slice, tokens c..c+15: silu(rs * gate) * (rs * up) -> bf16 into
  // the K-major activation tile (token rows of 128 bytes per 64-feature half, 16-byte chunks
  // swizzled by row % 8)
  if (acc_ok) {
    uint8_t* act = smem + kMlpOffAct + (tl >> 6) * kMlpXBlk;
    const int e = tl & 63;
#pragma unroll 1
    for (int c = hh * 16; c < nv; c += 16 * (kMlpThreads / 128)) {
      uint32_t g[16], u[16];
      tmem_ld16(lane_addr + c, g);
      tmem_ld16(lane_addr + 64 + c, u);
      tmem_ld_wait(g, u);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int tok = c + j;
        const float rs = rtab[tok < 64 ? tok : 0];
        const float v = silu(__uint_as_float(g[j]) * rs) * (__uint_as_float(u[j]) * rs);
        *reinterpret_cast<__nv_bfloat16*>(act + tok * 128 + (((e >> 3) ^ (tok & 7)) << 4) + (e & 7) * 2) =
            __float2bfloat16_rn(v);
      }
    }
  }
  mlp_fence_async_smem();  // the activation tile's generic-proxy stores, before the MMA reads them
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    // warp 0 waits together, its elected lane issues (warp-uniform descriptors)
    if (acc_ok && __all_sync(0xffffffffu, mbar_wait(down_full, 0, a.status))) {
      tc_fence_after();
      if (elect_one()) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint64_t ad = sw128_desc(smem_u32(smem + kMlpOffDown + h * kMlpWBlk));
          const uint64_t bd = sw128_desc(smem_u32(smem + kMlpOffAct + h * kMlpXBlk));
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f16(tmem + 128, ad + 2 * k, bd + 2 * k, kIdesc, (h > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(down_done);
      }
    } else if (elect_one()) {
      mbar_arrive(down_done);
    }
  }
  __syncwarp();
  const bool down_ok = __all_sync(0xffffffffu, mbar_wait(down_done, 0, a.status) ? 1 : 0) != 0;
  tc_fence_after();

  // this CTA's partial of the output tile, token-major over the (idle) ring
  float* part = reinterpret_cast<float*>(smem);
  if (down_ok) {
#pragma unroll 1
    for (int c = hh * 16; c < nv; c += 16 * (kMlpThreads / 128)) {
      uint32_t d[16];
      tmem_ld16(lane_addr + 128 + c, d);
      tmem_ld_wait(d);
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(c + j) * 128 + tl] = __uint_as_float(d[j]);
    }
  }
  tc_fence_before();
  cluster_sync();
  cluster_token_reduce<kMlpMaxCluster, kMlpThreads>(a.ep, part, static_cast<int>(gridDim.x), nv, row0, tile, pf);
  cluster_sync_relaxed();  // no CTA leaves while a peer still reads its partial
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

}  // namespace so101

using namespace so101;

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

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// bf16 K-major map: rows x inner elements, row stride ld, boxes of 64 x box_rows (SWIZZLE_128B).
int map_bf16(CUtensorMap* m, const void* p, long long inner, long long rows, long long ld, int box_rows) {
  EncodeFn enc = encode_fn();
  if (!enc) return SO101_ERR_DRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(p), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? SO101_OK
             : SO101_ERR_ARG;
}

// Whether a cluster of `size` CTAs of the kernel can be resident at all (sizes above 8 are
// non-portable and depend on the GPU); cached per size.
int cluster_fits(int size, cudaStream_t stream) {
  static int known[kMlpMaxCluster + 1] = {};  // 0 unknown, 1 fits, -1 does not
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(mlp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMlpSmem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(mlp_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  if (known[size] == 0) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(size, 1, 1);
    lc.blockDim = dim3(kMlpThreads);
    lc.dynamicSmemBytes = kMlpSmem;
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int clusters = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, mlp_kernel, &lc);
    if (e != cudaSuccess) return launch_error(e);
    known[size] = clusters > 0 ? 1 : -1;
  }
  return known[size] > 0 ? SO101_OK : SO101_ERR_ARG;
}

}  // namespace

extern "C" int so101_mlp(const void* x, int64_t ldx, int64_t rows, int batch, int64_t k, const float* rms_ss,
                         int rms_slots, int64_t rms_ld, float rms_eps, const void* w_gate_up, int64_t ldw1, int64_t mlp,
                         const void* w_down, int64_t ldw2, int64_t n_out, float* y, int64_t ldy, const float* residual,
                         int64_t ldr, void* y16, int64_t ld16, const float* y16_scale, float* stat_ss,
                         int64_t stat_ld, cudaStream_t stream) {
  if (!x || !w_gate_up || !w_down || !y || rows <= 0 || rows > 64 || batch <= 0 || batch > 65535 || k <= 0)
    return SO101_ERR_ARG;
  if (mlp <= 0 || mlp % 128 || mlp / 128 > kMlpMaxCluster || n_out <= 0 || n_out % 4 || n_out > (1 << 20))
    return SO101_ERR_ARG;
  if (k > (1 << 20) || static_cast<long long>(batch) * rows > (1 << 30)) return SO101_ERR_ARG;
  if (rms_ss && (rms_slots < 1 || rms_slots > 64 || rms_ld < rms_slots)) return SO101_ERR_ARG;
  // TMA: 16-byte bases and row strides
  if (!aligned16(x) || !aligned16(w_gate_up) || !aligned16(w_down) || (ldx * 2) % 16 || (ldw1 * 2) % 16 ||
      (ldw2 * 2) % 16 || ldx < k || ldw1 < k || ldw2 < mlp)
    return SO101_ERR_ARG;
  if (!aligned16(y) || ldy % 4 || ldy < n_out) return SO101_ERR_ARG;
  if (residual && (!aligned16(residual) || ldr % 4 || ldr < n_out)) return SO101_ERR_ARG;
  if (y16 && (reinterpret_cast<uintptr_t>(y16) % 8 || ld16 % 4 || ld16 < n_out)) return SO101_ERR_ARG;
  if (y16_scale && !aligned16(y16_scale)) return SO101_ERR_ARG;
  const int tiles = static_cast<int>((n_out + 127) / 128);
  if (tiles > 65535 || (stat_ss && stat_ld < tiles)) return SO101_ERR_ARG;

  CUtensorMap tx, tgu, td;
  int rc = map_bf16(&tx, x, k, static_cast<long long>(batch) * rows, ldx, 64);
  if (rc == SO101_OK) rc = map_bf16(&tgu, w_gate_up, k, 2 * mlp, ldw1, 128);
  if (rc == SO101_OK) rc = map_bf16(&td, w_down, mlp, n_out, ldw2, 128);
  if (rc != SO101_OK) return rc;
  const int S = static_cast<int>(mlp / 128);
  rc = cluster_fits(S, stream);
  if (rc != SO101_OK) return rc;

  MlpArgs a;
  a.ep = TokenEpilogue{y, ldy, residual, ldr, static_cast<__nv_bfloat16*>(y16), ld16, y16_scale, stat_ss, stat_ld,
                       static_cast<int>(n_out)};
  a.rows = static_cast<int>(rows);
  a.kb = static_cast<int>((k + 63) / 64);
  a.mlp = static_cast<int>(mlp);
  a.rms_ss = rms_ss;
  a.rms_slots = rms_slots;
  a.rms_ld = rms_ld;
  a.rms_n = static_cast<float>(k);
  a.rms_eps = rms_eps;
  a.status = status_ptr();

  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(S, tiles, batch);
  lc.blockDim = dim3(kMlpThreads);
  lc.dynamicSmemBytes = kMlpSmem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&lc, mlp_kernel, tx, tgu, td, a);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}
