// Attention fused with its output projection and residual, for the few query rows of the action
// expert at batch 1: y = residual + attention(q, k, v) @ W_o^T, one launch instead of an attention
// launch followed by a GEMM launch.
//
// The output projection's K dimension is the heads: y = sum over heads h of O_h W_o[:, h]^T, with
// O_h the (rows x 64) attention output of head h and W_o[:, h] the 64 columns of W_o that read it.
// So the grid is clusters of nq CTAs (one per query head, cluster rank = head) per 128-feature
// output tile and 64-row query block. Each CTA
//   1  issues the TMA load of its W_o block (128 features x 64, SWIZZLE_128B) before waiting for
//      the previous grid: the weights do not depend on it;
//   2  runs the flash attention of its head over all key tiles (attention_tile.cuh; a six-tile K/V
//      ring, so the expert's 291 keys arrive in one round of loads; two or three warp groups
//      taking the tiles in turn, whichever needs fewer rounds, merged at the end), writing the
//      normalised rows as bf16 straight into the MMA's B operand tile in shared memory (the same
//      bf16 rounding the unfused path applies before storing them);
//   3  issues one M=128, N=64, K=64 tcgen05.mma: its head's fp32 partial (features x tokens) in
//      TMEM, staged to shared memory;
//   4  after a cluster barrier, sums whole tokens over the nq partials through DSMEM in head
//      order and runs the residual epilogue (token_reduce.cuh): fp32 row, bf16 copy scaled by the
//      next RMSNorm's weight, the token's sum of squares over the tile (statistics slot = tile).
// Redundancy: every output tile's cluster recomputes the attention (a few microseconds of tensor
// work on the key/value rows that L2 holds); what it saves is a dependent launch and the round
// trip of the attention output through global memory.
#include <mutex>

#include "attention_tile.cuh"
#include "token_reduce.cuh"

namespace so101 {

struct AttnOArgs {
  AttnArgs at;       // at.o unused
  TokenEpilogue ep;  // output tile epilogue
  int q_blocks;      // 64-row query blocks per problem
  int* status;
};

constexpr int kAoBuf = 6;                               // K/V ring: the expert's 5 key tiles at once
constexpr int kAoMaxHeads = 16;                         // largest (non-portable) cluster
constexpr int kAoOffW = 0;                              // W_o block: 128 x 64 bf16, 16 KB
constexpr int kAoOffO = 128 * 128;                      // O tile: 64 x 64 bf16, 8 KB
constexpr int kAoOffAttn = kAoOffO + 64 * 128;          // attention_body's area, then the partial
constexpr int kAoOffBar = kAoOffAttn + attention_smem_bytes<64, kAoBuf>();
constexpr int kAoSmem = kAoOffBar + 64 + 1024;          // + 1024-byte alignment of the base
static_assert(attention_smem_bytes<64, kAoBuf>() >= 64 * 128 * 4, "the fp32 partial reuses the attention area");

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// G warp groups of 128 threads take the key tiles in turn (attention_body's WG).
template <int G>
__global__ void __launch_bounds__(128 * G, 1) attention_o_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                 const AttnOArgs a) {
  constexpr int kAoThreads = 128 * G;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + kAoOffBar);
  uint64_t* mma_done = w_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  const int t = threadIdx.x, warp = t >> 5;
  const int h = blockIdx.x, tile = blockIdx.y;
  const int qb = blockIdx.z % a.q_blocks, bi = blockIdx.z / a.q_blocks;
  const int q0 = qb * 64;
  constexpr uint32_t kCols = 64;

  if (t == 0) {
    mbar_init(w_full, 1);
    mbar_init(mma_done, 1);
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
  if (t == 0) {
    tma_prefetch_desc(&tm_w);
    mbar_arrive_expect_tx(w_full, 128 * 128);
    tma_load_2d(smem + kAoOffW, &tm_w, w_full, h * 64, tile * 128, policy_evict_normal());
  }
  grid_dep_launch();
  grid_dep_wait();
  const int nv = min(64, a.at.Lq - q0);  // valid tokens of this query block
  const long long row0 = static_cast<long long>(bi) * a.at.Lq + q0;
  const TokenPrefetch pf = token_prefetch<kAoThreads>(a.ep, a.at.nq, nv, row0, tile);

  attention_body<64, false, true, kAoBuf, G>(a.at, 0, q0, h, bi, smem + kAoOffAttn, smem + kAoOffO);
  fence_async_smem();  // the O tile's generic-proxy stores, before the tensor core reads them
  __syncthreads();
  if (t == 0) {
    if (mbar_wait(w_full, 0, a.status)) {
      tc_fence_after();
      const uint64_t ad = sw128_desc(smem_u32(smem + kAoOffW)), bd = sw128_desc(smem_u32(smem + kAoOffO));
#pragma unroll
      for (int k = 0; k < 4; ++k) mma_f16(tmem, ad + 2 * k, bd + 2 * k, idesc_bf16(128, 64), k > 0 ? 1u : 0u);
      mma_commit(mma_done);
    } else {
      mbar_arrive(mma_done);  // the weights never came: unwind through the cluster barriers
    }
  }
  __syncwarp();
  const bool mma_ok = __all_sync(0xffffffffu, mbar_wait(mma_done, 0, a.status) ? 1 : 0) != 0;
  tc_fence_after();

  // this head's partial, column-major (a token's 128 features contiguous), over the attention area
  float* part = reinterpret_cast<float*>(smem + kAoOffAttn);
  if (mma_ok) {
    // thread t: TMEM lane t % 128 (warp w reads lanes 32 (w % 4) ..), 16-token chunks c with
    // c / 16 = t / 128 modulo the group count
    const int tl = t & 127;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll 1
    for (int c = (t >> 7) * 16; c < nv; c += 16 * G) {
      uint32_t r[16];
      tmem_ld16(lane_addr + c, r);
      tmem_ld_wait(r);
#pragma unroll
      for (int j = 0; j < 16; ++j) part[(c + j) * 128 + tl] = __uint_as_float(r[j]);
    }
  }
  tc_fence_before();
  cluster_sync();

  cluster_token_reduce<kAoMaxHeads, kAoThreads>(a.ep, part, a.at.nq, nv, row0, tile, pf);
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

// Whether a cluster of `heads` CTAs of attention_o_kernel<G> can be resident at all (non-portable
// sizes above 8 depend on the GPU); cached per group count and cluster size.
template <int G>
int cluster_fits(int heads, cudaStream_t stream) {
  static int known[kAoMaxHeads + 1] = {};  // 0 unknown, 1 fits, -1 does not
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_o_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAoSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(attention_o_kernel<G>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  if (known[heads] == 0) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(heads, 1, 1);
    lc.blockDim = dim3(128 * G);
    lc.dynamicSmemBytes = kAoSmem;
    lc.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = heads;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int clusters = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, attention_o_kernel<G>, &lc);
    if (e != cudaSuccess) return launch_error(e);
    known[heads] = clusters > 0 ? 1 : -1;
  }
  return known[heads] > 0 ? SO101_OK : SO101_ERR_ARG;
}

}  // namespace

extern "C" int so101_attention_o(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                 int64_t Lq, int64_t Lk, int nq, int nkv, int hd, int64_t causal_from,
                                 int64_t q_offset, const float* cos, const float* sin, int batch, int64_t bq,
                                 int64_t bk, int64_t bv, const void* k_own, const void* v_own, int64_t ld_own,
                                 int64_t b_own, int64_t own_from, const float* k_cos, const float* k_sin,
                                 const void* w_o, int64_t ldw, int64_t n_out, float* y, int64_t ldy,
                                 const float* residual, int64_t ldr, void* y16, int64_t ld16, const float* y16_scale,
                                 float* stat_ss, int64_t stat_ld, cudaStream_t stream) {
  if (!q || !k || !v || !w_o || !y || Lq <= 0 || Lk <= 0 || nkv <= 0 || nq <= 0 || nq % nkv || batch <= 0)
    return SO101_ERR_ARG;
  if (hd != 64 || nq > kAoMaxHeads || n_out <= 0 || n_out % 4 || n_out > (1 << 20)) return SO101_ERR_ARG;
  if (Lq > (1 << 24) || Lk > (1 << 30)) return SO101_ERR_ARG;
  if ((cos == nullptr) != (sin == nullptr)) return SO101_ERR_ARG;
  const long long q_blocks = (Lq + 63) / 64;
  if (q_blocks * batch > 65535 || (n_out + 127) / 128 > 65535) return SO101_ERR_ARG;
  // attention operands, as so101_attention checks them
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (ldq * 2) % 16 || (ldk * 2) % 16 || (ldv * 2) % 16 ||
      (bq * 2) % 16 || (bk * 2) % 16 || (bv * 2) % 16)
    return SO101_ERR_ARG;
  if (cos && (!aligned16(cos) || !aligned16(sin))) return SO101_ERR_ARG;
  if (k_own) {
    if (!v_own || !k_cos || !k_sin || own_from < 0 || own_from > Lk || !aligned16(k_own) || !aligned16(v_own) ||
        (ld_own * 2) % 16 || (b_own * 2) % 16)
      return SO101_ERR_ARG;
  }
  // projection and epilogue: 16-byte weight rows for TMA, float4 / 4 x bf16 row pieces
  if (!aligned16(w_o) || (ldw * 2) % 16 || ldw < static_cast<int64_t>(nq) * hd) return SO101_ERR_ARG;
  if (!aligned16(y) || ldy % 4 || ldy < n_out) return SO101_ERR_ARG;
  if (residual && (!aligned16(residual) || ldr % 4 || ldr < n_out)) return SO101_ERR_ARG;
  if (y16 && (reinterpret_cast<uintptr_t>(y16) % 8 || ld16 % 4 || ld16 < n_out)) return SO101_ERR_ARG;
  if (y16_scale && !aligned16(y16_scale)) return SO101_ERR_ARG;
  const int tiles = static_cast<int>((n_out + 127) / 128);
  if (stat_ss && stat_ld < tiles) return SO101_ERR_ARG;

  EncodeFn enc = encode_fn();
  if (!enc) return SO101_ERR_DRIVER;
  CUtensorMap tm;
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(nq) * hd, static_cast<cuuint64_t>(n_out)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldw) * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t estr[2] = {1, 1};
    if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w_o), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return SO101_ERR_ARG;
  }
  // key tiles of the last query block (attention_body's count): three warp groups when that takes
  // fewer rounds than two (the expert's 291 self-attention keys: 5 tiles, 2 rounds against 3)
  long long last = causal_from - 1;
  if ((q_blocks - 1) * 64 + 63 + q_offset > last) last = (q_blocks - 1) * 64 + 63 + q_offset;
  if (last > Lk - 1) last = Lk - 1;
  const long long key_tiles = (last + 64) / 64;
  const int groups = (key_tiles + 2) / 3 < (key_tiles + 1) / 2 ? 3 : 2;
  const int fit = groups == 3 ? cluster_fits<3>(nq, stream) : cluster_fits<2>(nq, stream);
  if (fit != SO101_OK) return fit;

  AttnOArgs a;
  AttnArgs& at = a.at;
  at.q = static_cast<const __nv_bfloat16*>(q);
  at.k = static_cast<const __nv_bfloat16*>(k);
  at.v = static_cast<const __nv_bfloat16*>(v);
  at.o = nullptr;
  at.ldq = ldq;
  at.ldk = ldk;
  at.ldv = ldv;
  at.ldo = 0;
  at.bq = bq;
  at.bk = bk;
  at.bv = bv;
  at.bo = 0;
  at.o_type = SO101_BF16;
  at.o_qscale = 0.f;
  at.Lq = static_cast<int>(Lq);
  at.Lk = static_cast<int>(Lk);
  at.nq = nq;
  at.nkv = nkv;
  at.causal_from = causal_from;
  at.q_offset = q_offset;
  at.cos = cos;
  at.sin = sin;
  at.scale_log2 = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(hd)));
  at.kv_splits = 1;
  at.k_own = static_cast<const __nv_bfloat16*>(k_own);
  at.v_own = static_cast<const __nv_bfloat16*>(v_own);
  at.ld_own = ld_own;
  at.b_own = b_own;
  at.own_from = own_from;
  at.k_cos = k_cos;
  at.k_sin = k_sin;
  a.ep = TokenEpilogue{y, ldy, residual, ldr, static_cast<__nv_bfloat16*>(y16), ld16, y16_scale, stat_ss, stat_ld,
                       static_cast<int>(n_out)};
  a.q_blocks = static_cast<int>(q_blocks);
  a.status = status_ptr();

  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(nq, tiles, static_cast<unsigned>(q_blocks * batch));
  lc.blockDim = dim3(128 * groups);
  lc.dynamicSmemBytes = kAoSmem;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nq;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = groups == 3 ? cudaLaunchKernelEx(&lc, attention_o_kernel<3>, tm, a)
                                    : cudaLaunchKernelEx(&lc, attention_o_kernel<2>, tm, a);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}
