// Grouped-query attention entry point: the tcgen05 kernels for the unmasked equal-length SigLIP
// case (attention_tc.cu) and for the masked prefix / expert attention over many observations
// (attention_gqa_tc.cu), the mma.sync flash attention (attention_tile.cuh) for everything else
// (few CTAs, where it splits the keys over a cluster, and the step's own keys rotated on chip).
#include <cstdlib>

#include "attention_tile.cuh"

namespace so101 {

template <int HD>
int launch_attention(const AttnArgs& a, int batch, cudaStream_t stream) {
  constexpr int smem = attention_smem_bytes<HD>();
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
bool attention_gqa_tc_eligible(const void* q, long long ldq, const void* k, long long ldk, const void* v,
                               long long ldv, const void* o, long long ldo, int o_type, long long Lq, long long Lk,
                               int nq, int nkv, int hd, const float* cos, long long bq, long long bk, long long bv,
                               long long bo, int batch, const void* k_own, const void* v_own, long long ld_own,
                               long long b_own, long long own_from, const float* k_cos, const float* k_sin);
int attention_gqa_tc_launch(const void* q, long long ldq, const void* k, long long ldk, const void* v, long long ldv,
                            void* o, long long ldo, long long Lq, long long Lk, int nq, int nkv,
                            long long causal_from, long long q_offset, const float* cos, const float* sin, int batch,
                            long long bq, long long bk, long long bv, long long bo, const void* k_own,
                            const void* v_own, long long ld_own, long long b_own, long long own_from,
                            const float* k_cos, const float* k_sin, cudaStream_t stream);

// The masked tcgen05 kernel for many observations; SO101_ATTN_GQA_TC=0 keeps the mma.sync kernel
// (for comparisons).
bool gqa_tc_enabled() {
  static const bool on = [] {
    const char* e = getenv("SO101_ATTN_GQA_TC");
    return !(e && e[0] == '0');
  }();
  return on;
}

}  // namespace so101

using namespace so101;

namespace {

struct OwnRows {
  const void* k;
  const void* v;
  int64_t ld, b, from;
  const float* cos;
  const float* sin;
};

int attention_impl(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                   int64_t ldo, int o_type, float o_qscale, int64_t Lq, int64_t Lk, int nq, int nkv, int hd,
                   int64_t causal_from, int64_t q_offset, const float* cos, const float* sin, int batch, int64_t bq,
                   int64_t bk, int64_t bv, int64_t bo, const OwnRows& own, cudaStream_t stream) {
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
  if (own.k) {  // the step's own keys and values from the fused qkv rows, keys rotated on chip
    if (!own.v || !own.cos || !own.sin || own.from < 0 || own.from > Lk || hd != 64) return SO101_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(own.k) % 16 || reinterpret_cast<uintptr_t>(own.v) % 16 || (own.ld * 2) % 16 ||
        (own.b * 2) % 16)
      return SO101_ERR_ARG;
  }
  if (!own.k &&
      attention_tc_eligible(q, ldq, k, ldk, v, ldv, Lq, Lk, nq, nkv, hd, causal_from, cos, bq, bk, bv, o_type) &&
      ldo % 8 == 0 && bo == Lq * ldo && reinterpret_cast<uintptr_t>(o) % 16 == 0)
    return attention_tc_launch(q, ldq, k, ldk, v, ldv, o, ldo, o_type, o_qscale, Lq, nq, batch, stream);
  if (gqa_tc_enabled() &&
      attention_gqa_tc_eligible(q, ldq, k, ldk, v, ldv, o, ldo, o_type, Lq, Lk, nq, nkv, hd, cos, bq, bk, bv, bo,
                                batch, own.k, own.v, own.ld, own.b, own.from, own.cos, own.sin))
    return attention_gqa_tc_launch(q, ldq, k, ldk, v, ldv, o, ldo, Lq, Lk, nq, nkv, causal_from, q_offset, cos, sin,
                                   batch, bq, bk, bv, bo, own.k, own.v, own.ld, own.b, own.from, own.cos, own.sin,
                                   stream);
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
  a.k_own = static_cast<const __nv_bfloat16*>(own.k);
  a.v_own = static_cast<const __nv_bfloat16*>(own.v);
  a.ld_own = own.ld;
  a.b_own = own.b;
  a.own_from = own.from;
  a.k_cos = own.cos;
  a.k_sin = own.sin;
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

}  // namespace

extern "C" int so101_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                               void* o, int64_t ldo, int o_type, float o_qscale, int64_t Lq, int64_t Lk, int nq,
                               int nkv, int hd, int64_t causal_from, int64_t q_offset, const float* cos,
                               const float* sin, int batch, int64_t bq, int64_t bk, int64_t bv, int64_t bo,
                               cudaStream_t stream) {
  return attention_impl(q, ldq, k, ldk, v, ldv, o, ldo, o_type, o_qscale, Lq, Lk, nq, nkv, hd, causal_from, q_offset,
                        cos, sin, batch, bq, bk, bv, bo, OwnRows{}, stream);
}

extern "C" int so101_attention_rows(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                    void* o, int64_t ldo, int o_type, float o_qscale, int64_t Lq, int64_t Lk, int nq,
                                    int nkv, int hd, int64_t causal_from, int64_t q_offset, const float* cos,
                                    const float* sin, int batch, int64_t bq, int64_t bk, int64_t bv, int64_t bo,
                                    const void* k_own, const void* v_own, int64_t ld_own, int64_t b_own,
                                    int64_t own_from, const float* k_cos, const float* k_sin, cudaStream_t stream) {
  if (!k_own) return SO101_ERR_ARG;
  return attention_impl(q, ldq, k, ldk, v, ldv, o, ldo, o_type, o_qscale, Lq, Lk, nq, nkv, hd, causal_from, q_offset,
                        cos, sin, batch, bq, bk, bv, bo, OwnRows{k_own, v_own, ld_own, b_own, own_from, k_cos, k_sin},
                        stream);
}
