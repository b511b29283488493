// Flash attention on tcgen05 for the unmasked, equal-length case (SigLIP: 1024 tokens per image,
// 12 heads of 64, no RoPE): the vision tower's dominant kernel at batch 64.
//
// One CTA = 256 query rows of one (image, head), as two groups of 128 (MMA M = 128). Per 128-key
// tile j:
//   warp 0 (one thread)  TMA: Q once, then K_j and V_j into a two-stage ring
//   warp 1 (one thread)  S_g = Q_g K_j^T  (M 128, N 128, K 64)       -> TMEM S_g
//                        O_g = P_g V_j    (M 128, N 64,  K 128 keys) -> TMEM O_g, fresh per tile
//   warps 2-5 / 6-9      softmax for group A / B, one thread per query row (its TMEM lane): the
//                        row's 128 scores are read twice from TMEM (max, then exp2), P goes to
//                        shared memory as bf16 in the swizzled K-major layout the MMA reads, and
//                        O_j is folded into a register accumulator with the running-max rescale.
// K and Q are K-major operands (head dim contiguous); V is an MN-major operand (head dim
// contiguous along N, keys along K) straight from its TMA tile. Softmax in fp32 with exp2 on
// log2(e)/sqrt(d)-scaled scores, P rounded to bf16 for P V, row sums from the fp32 P.
#include "common.cuh"

namespace so101 {

struct AttnTcArgs {
  void* o;
  long long ldo;
  int o_type;
  float o_qinv;
  int L;            // tokens per image (queries = keys)
  float scale_log2;
  int* status;
};

constexpr int kTcRows = 128;   // rows per group (MMA M)
constexpr int kTcKeys = 128;   // keys per tile (MMA N of S, K of P V)
constexpr int kTcHd = 64;
constexpr int kTcTile = kTcRows * kTcHd * 2;   // 16 KB: a 128 x 64 bf16 tile
constexpr int kTcThreads = 320;

// smem offsets (from a 1024-aligned base)
constexpr int kOffQ = 0;                          // 2 groups x 16 KB
constexpr int kOffK = kOffQ + 2 * kTcTile;        // 2 stages x 16 KB
constexpr int kOffV = kOffK + 2 * kTcTile;        // 2 stages x 16 KB
constexpr int kOffP = kOffV + 2 * kTcTile;        // 2 groups x 32 KB (two 64-key halves each)
constexpr int kOffBar = kOffP + 4 * kTcTile;
constexpr int kTcSmem = kOffBar + 256 + 1024;

// TMEM columns: S_A, S_B (128 each), O_A, O_B (64 each)
constexpr uint32_t kColS = 0, kColO = 256;

// Instruction descriptor: bf16 A/B, fp32 D, A K-major, B K-major (b_mn = 0) or MN-major (1).
__host__ __device__ constexpr uint32_t idesc_attn(int n, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(b_mn) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(128 >> 4) << 24);
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two floats rounded to bf16 (nearest even) and packed, the first in the low half.
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(kTcThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const AttnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bar;           // [1]
  uint64_t* kv_full = bar + 1;      // [2]
  uint64_t* kv_empty = bar + 3;     // [2]
  uint64_t* s_full = bar + 5;       // [2] per group
  uint64_t* s_free = bar + 7;       // [2]
  uint64_t* p_full = bar + 9;       // [2]
  uint64_t* o_full = bar + 11;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 13);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y, img = blockIdx.z;
  const int row0 = img * a.L + blockIdx.x * 2 * kTcRows;  // first query row (global token row)
  const int key0 = img * a.L;
  const int n_tiles = a.L / kTcKeys;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
    fence_mbar_init();
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
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      grid_dep_wait();
      const uint64_t keep = policy_evict_last();
      const int xq = head * kTcHd;
      mbar_arrive_expect_tx(q_full, 2 * kTcTile);
      tma_load_2d(smem + kOffQ, &tm_q, q_full, xq, row0, keep);
      tma_load_2d(smem + kOffQ + kTcTile, &tm_q, q_full, xq, row0 + kTcRows, keep);
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1u, a.status)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTcTile);
        tma_load_2d(smem + kOffK + st * kTcTile, &tm_k, &kv_full[st], xq, key0 + j * kTcKeys, keep);
        tma_load_2d(smem + kOffV + st * kTcTile, &tm_v, &kv_full[st], xq, key0 + j * kTcKeys, keep);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_attn(kTcKeys, 0);
      constexpr uint32_t ID_O = idesc_attn(kTcHd, 1);
      bool ok = mbar_wait(q_full, 0, a.status);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1u, a.status)) break;
        tc_fence_after();
        const uint32_t kaddr = smem_u32(smem + kOffK + st * kTcTile);
        const uint32_t vaddr = smem_u32(smem + kOffV + st * kTcTile);
        for (int g = 0; g < 2; ++g) {
          if (j >= 1 && !mbar_wait(&s_free[g], (j - 1) & 1u, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t qd = sw128_desc(smem_u32(smem + kOffQ + g * kTcTile));
          const uint64_t kd = sw128_desc(kaddr);
#pragma unroll
          for (int k = 0; k < kTcHd / 16; ++k)
            mma_f16(tmem + kColS + g * kTcKeys, qd + 2 * k, kd + 2 * k, ID_S, k > 0 ? 1u : 0u);
          mma_commit(&s_full[g]);
        }
        if (!ok) break;
        for (int g = 0; g < 2; ++g) {
          if (!mbar_wait(&p_full[g], j & 1u, a.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t paddr = smem_u32(smem + kOffP + g * 2 * kTcTile);
          const uint64_t vd = sw128_desc(vaddr);
#pragma unroll
          for (int k = 0; k < kTcKeys / 16; ++k) {
            // P: keys [16k, 16k+16) sit in the (k / 4)-th 64-key half, 32 bytes per step within it;
            // V (MN-major): 16 keys = two 8-row groups = 2048 bytes per step
            const uint64_t pd = sw128_desc(paddr + (k >> 2) * kTcTile) + 2 * (k & 3);
            mma_f16(tmem + kColO + g * kTcHd, pd, vd + static_cast<uint64_t>(k) * (2048 >> 4), ID_O,
                    k > 0 ? 1u : 0u);
          }
          mma_commit(&o_full[g]);
        }
        mma_commit(&kv_empty[st]);
      }
    }
  } else {
    // ---------------- softmax: group g = (warp - 2) / 4, row r = quad * 32 + lane
    grid_dep_wait();
    const int g = (warp - 2) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_addr = lane_base + kColS + g * kTcKeys;
    const uint32_t o_addr = lane_base + kColO + g * kTcHd;
    uint8_t* P = smem + kOffP + g * 2 * kTcTile;
    float m = -INFINITY, l = 0.f;
    float acc[kTcHd];
#pragma unroll
    for (int d = 0; d < kTcHd; ++d) acc[d] = 0.f;
    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait(&s_full[g], j & 1u, a.status)) break;
      tc_fence_after();
      // pass 1: the tile's row maximum
      float tmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < kTcKeys; c += 32) {
        uint32_t v0[16], v1[16];
        tmem_ld16(s_addr + c, v0);
        tmem_ld16(s_addr + c + 16, v1);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) tmax = fmaxf(tmax, fmaxf(__uint_as_float(v0[e]), __uint_as_float(v1[e])));
      }
      const float m_new = fmaxf(m, tmax * a.scale_log2);
      const float alpha = ex2(m - m_new);
      // pass 2: P = exp2(s * scale - m_new) as bf16 into the swizzled K-major tile, row sums in fp32
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < kTcKeys; c += 32) {
        uint32_t v0[16], v1[16];
        tmem_ld16(s_addr + c, v0);
        tmem_ld16(s_addr + c + 16, v1);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float p0 = ex2(fmaf(__uint_as_float(v0[2 * e]), a.scale_log2, -m_new));
          const float p1 = ex2(fmaf(__uint_as_float(v0[2 * e + 1]), a.scale_log2, -m_new));
          const float p2 = ex2(fmaf(__uint_as_float(v1[2 * e]), a.scale_log2, -m_new));
          const float p3 = ex2(fmaf(__uint_as_float(v1[2 * e + 1]), a.scale_log2, -m_new));
          lsum += (p0 + p1) + (p2 + p3);
          pk[e] = bf16x2(p0, p1);
          pk[8 + e] = bf16x2(p2, p3);
        }
        // keys c .. c+31 = four 16-byte chunks of row r in half c / 64, chunk (c % 64) / 8 + i
        uint8_t* rowp = P + (c >> 6) * kTcTile + (r >> 3) * 1024 + (r & 7) * 128;
        const int ch = (c & 63) >> 3;  // first of this row's four 16-byte chunks
        *reinterpret_cast<uint4*>(rowp + (((ch + 0) ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(rowp + (((ch + 1) ^ (r & 7)) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        *reinterpret_cast<uint4*>(rowp + (((ch + 2) ^ (r & 7)) << 4)) = make_uint4(pk[8], pk[9], pk[10], pk[11]);
        *reinterpret_cast<uint4*>(rowp + (((ch + 3) ^ (r & 7)) << 4)) = make_uint4(pk[12], pk[13], pk[14], pk[15]);
      }
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_free[g]);
        mbar_arrive(&p_full[g]);
      }
      l = l * alpha + lsum;
      m = m_new;
      // O += alpha-rescaled previous + this tile's P V
      if (!mbar_wait(&o_full[g], j & 1u, a.status)) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < kTcHd; c += 16) {
        uint32_t ov[16];
        tmem_ld16(o_addr + c, ov);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[c + e] = fmaf(acc[c + e], alpha, __uint_as_float(ov[e]));
      }
    }
    // write O / l for this row
    const float inv = 1.f / l;
    const long long orow = row0 + g * kTcRows + r;
    if (a.o_type == SO101_BF16) {
      uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.o) + orow * a.ldo + head * kTcHd);
#pragma unroll
      for (int q = 0; q < kTcHd / 8; ++q) {
        const float* v = acc + 8 * q;
        dst[q] = make_uint4(bf16x2(v[0] * inv, v[1] * inv), bf16x2(v[2] * inv, v[3] * inv),
                            bf16x2(v[4] * inv, v[5] * inv), bf16x2(v[6] * inv, v[7] * inv));
      }
    } else {
      uint4* dst = reinterpret_cast<uint4*>(static_cast<int8_t*>(a.o) + orow * a.ldo + head * kTcHd);
#pragma unroll
      for (int q = 0; q < kTcHd / 16; ++q) {
        const float* v = acc + 16 * q;
        dst[q] = make_uint4(pack4_i8(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv, a.o_qinv),
                            pack4_i8(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv, a.o_qinv),
                            pack4_i8(v[8] * inv, v[9] * inv, v[10] * inv, v[11] * inv, a.o_qinv),
                            pack4_i8(v[12] * inv, v[13] * inv, v[14] * inv, v[15] * inv, a.o_qinv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

namespace {

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// rows x 64-column boxes over a bf16 matrix of `rows` rows with row stride ld elements; the map's
// inner extent stops at `cols` so a box never reads past the head it starts in.
int map_rows(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld) {
  EncodeFn enc = encode();
  if (!enc) return SO101_ERR_DRIVER;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? SO101_OK
             : SO101_ERR_ARG;
}

}  // namespace

// Whether the tcgen05 kernel serves this problem, and its launch.
bool attention_tc_eligible(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                           long long Lq, long long Lk, int nq, int nkv, int hd, long long causal_from,
                           const float* cos, long long bq, long long bk, long long bv, int o_type) {
  return hd == 64 && nq == nkv && Lq == Lk && Lq % 256 == 0 && causal_from >= Lk && !cos && bq == Lq * ldq &&
         bk == Lk * ldk && bv == Lk * ldv && (ldq * 2) % 16 == 0 && (ldk * 2) % 16 == 0 && (ldv * 2) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(v) % 16 == 0 && (o_type == SO101_BF16 || o_type == SO101_I8);
}

int attention_tc_launch(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                        void* o, long long ldo, int o_type, float o_qscale, long long L, int heads, int batch,
                        cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  const long long rows = L * batch, cols = static_cast<long long>(heads) * 64;
  int rc = map_rows(&tq, q, rows, cols, ldq);
  if (!rc) rc = map_rows(&tk, k, rows, cols, ldk);
  if (!rc) rc = map_rows(&tv, v, rows, cols, ldv);
  if (rc) return rc;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
    if (e != cudaSuccess) return launch_error(e);
    configured = true;
  }
  AttnTcArgs a;
  a.o = o;
  a.ldo = ldo;
  a.o_type = o_type;
  a.o_qinv = o_type == SO101_I8 ? static_cast<float>(1.0 / static_cast<double>(o_qscale)) : 0.f;
  a.L = static_cast<int>(L);
  a.scale_log2 = static_cast<float>(1.4426950408889634 / 8.0);
  a.status = status_ptr();
  return launch_kernel(attention_tc_kernel, dim3(static_cast<unsigned>(L / 256), heads, batch), dim3(kTcThreads),
                       kTcSmem, stream, tq, tk, tv, a);
}

}  // namespace so101
