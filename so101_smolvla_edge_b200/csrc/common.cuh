// PTX helpers for sm_100a: mbarriers, TMA, tcgen05 (TMEM alloc, MMA, loads), bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/so101_b200.h"

namespace so101 {

// Kernels record the first SO101_ERR_* they hit into a device status word whose address the
// host passes in (status.cu owns it; so101_device_status() reads it).
__device__ __forceinline__ void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Host side: the device address of the status word on the current device.
int* status_ptr();

// Host side: whether launches carry the programmatic-dependent-launch attribute (so101_set_pdl).
bool pdl_enabled();

// Host side: remember the CUDA error behind an SO101_ERR_LAUNCH (so101_last_error reports it) and
// return that status.
int launch_error(cudaError_t e);

// Launch `kern` on `stream`, with programmatic dependent launch when enabled: the kernel may then
// start while the previous kernel on the stream drains, and waits (griddepcontrol.wait) before
// it touches that kernel's results. Returns SO101_OK or SO101_ERR_LAUNCH.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&lc, kern, static_cast<KArgs>(args)...);
  return e == cudaSuccess ? SO101_OK : launch_error(e);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of an mbarrier, giving up after ~2 s of wall time: the wait records
// SO101_ERR_TIMEOUT and returns false so the caller can unwind instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      record_error(status, SO101_ERR_TIMEOUT);
      return false;
    }
  }
}

// Cluster-scope variants, for barriers that other CTAs of the cluster arrive on remotely.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      record_error(status, SO101_ERR_TIMEOUT);
      return false;
    }
  }
}

// Arrive on the mbarrier at shared::cluster address `addr` (another CTA's, from mapa). Release at
// CTA scope: what it orders is this thread's tcgen05 loads (fenced before it), not memory that the
// other CTA reads, and a cluster-scope release costs a fence per arrive.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}

// ---------------------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of box (x: inner, y: outer) into shared memory, completing tx on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// As tma_load_2d, for a CTA pair: the transferred bytes complete on the mbarrier at shared::cluster
// address `bar` (either CTA of the pair; the pair's even CTA counts both CTAs' bytes).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.cta_group::2.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, both K-major. kind::f16 (bf16 in, fp32 acc).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::i8 (s8 in, s32 acc).
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// One lane of a converged warp (the lowest) gets true. Issuing tcgen05 MMAs from a warp that runs
// the whole control flow together, with the elected lane issuing, keeps the descriptors and TMEM
// addresses warp-uniform; a lane-0-only branch around the loop measured 4% slower on the SigLIP
// attention, whose MMAs are small.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Arrive on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// CTA pair (cta_group::2): one warp of each of the two CTAs allocates / frees together; the even
// CTA issues M = 256 MMAs whose A rows and B columns are split between the two CTAs' shared
// memory (same offsets), each CTA's TMEM receiving its own 128 rows of D.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at this shared-memory offset in both CTAs of the pair when every
// cta_group::2 MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: this thread's lane, columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// As tmem_ld_wait, tying the destination registers of the loads it waits for, so that no use of
// them is scheduled before the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[16], uint32_t (&s)[16]) {
  tmem_ld_wait(r);
  asm volatile(""
               : "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]),
                 "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]), "+r"(s[14]), "+r"(s[15])
               :
               : "memory");
}

// Shared-memory matrix descriptor for a K-major tile stored as TMA SWIZZLE_128B writes it:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset 1024), leading byte
// offset unused for swizzled K-major (encoded 1), version 1 (sm_100), layout SWIZZLE_128B (2).
// The tile base must be 1024-byte aligned; a K sub-block k * 32 bytes in is addressed by adding
// (k * 32) >> 4 to the start-address field.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: dense, D fp32 (c_format 1) from bf16 A and B (formats 1), both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// Dense, D s32 (c_format 2) from signed int8 A and B (formats 1), both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------------------------- PDL
// Programmatic dependent launch: wait for the previous grid's memory, allow the next grid to
// start its independent prologue.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The barrier that keeps a CTA's shared memory alive until its peers' DSMEM reads are done, at the
// end of a kernel: a peer uses every value it loaded before it arrives, so its reads have returned
// by then, and nothing else needs ordering. A release arrive would also wait for this CTA's global
// stores to complete (about 0.5 us more, measured), which the end of the grid does anyway.
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// Address of the same shared-memory offset in cluster CTA `rank`, and a load through it.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// ---------------------------------------------------------------------------------- numerics
// Epilogue math stays off the transcendental (XU) pipe except for one tanh.approx per element.

// tanh on the hardware approximation (max abs error ~2^-11, far below a bf16 or int8 step).
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;
  return 0.5f * x * (1.0f + tanh_fast(k0 * fmaf(0.044715f * x, x * x, x)));
}

// The same GELU in five FMA-pipe operations around the tanh: x * (k0 + k0 * 0.044715 * x^2).
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float t = tanh_fast(x * fmaf(x * x, 0.7978845608028654f * 0.044715f, 0.7978845608028654f));
  const float h = 0.5f * x;
  return fmaf(h, t, h);
}

// Packed fp32x2 arithmetic (sm_100): two independent round-to-nearest fp32 operations per
// instruction on (x, y) pairs, so results equal the scalar ones bit for bit.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^x on the MUFU unit (PTX ex2.approx.ftz: subnormal inputs and results flush to zero).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// gelu_tanh_fast on a pair, packed; same operations in the same order, same results.
__device__ __forceinline__ float2 gelu_tanh_fast2(float2 x) {
  const float2 p = ffma2(fmul2(x, x), make_float2(0.7978845608028654f * 0.044715f, 0.7978845608028654f * 0.044715f),
                         make_float2(0.7978845608028654f, 0.7978845608028654f));
  const float2 a = fmul2(x, p);
  const float2 t = make_float2(tanh_fast(a.x), tanh_fast(a.y));
  const float2 h = fmul2(make_float2(0.5f, 0.5f), x);
  return ffma2(h, t, h);
}

// Four values to packed int8 (clamp(round_half_even(v * inv), -128, 127)): the clamped product
// plus 1.5 * 2^23 holds the rounded integer in the low byte of its bit pattern.
__device__ __forceinline__ uint32_t pack4_i8(float a, float b, float c, float d, float inv) {
  const float2 m01 = fmul2(make_float2(a, b), make_float2(inv, inv));
  const float2 m23 = fmul2(make_float2(c, d), make_float2(inv, inv));
  const float2 r01 = fadd2(make_float2(fminf(fmaxf(m01.x, -128.f), 127.f), fminf(fmaxf(m01.y, -128.f), 127.f)),
                           make_float2(12582912.0f, 12582912.0f));
  const float2 r23 = fadd2(make_float2(fminf(fmaxf(m23.x, -128.f), 127.f), fminf(fmaxf(m23.y, -128.f), 127.f)),
                           make_float2(12582912.0f, 12582912.0f));
  return __byte_perm(__byte_perm(__float_as_uint(r01.x), __float_as_uint(r01.y), 0x0040),
                     __byte_perm(__float_as_uint(r23.x), __float_as_uint(r23.y), 0x0040), 0x5410);
}

// SiLU through sigmoid(x) = (1 + tanh(x / 2)) / 2.
__device__ __forceinline__ float silu(float x) { return 0.5f * x * (1.0f + tanh_fast(0.5f * x)); }

// int32 -> fp32 correctly rounded on the FMA pipe: v = hi * 2^16 + lo, each half converted exactly
// by adding it to the bit pattern of a power of two (1.5 * 2^23 for the signed high half, 2^23 for
// the unsigned low half), then one fused multiply-add rounds once.
__device__ __forceinline__ float i32_to_f32(int v) {
  const int hi = v >> 16;
  const int lo = v & 0xFFFF;
  const float fhi = __int_as_float(0x4B400000 + hi) - 12582912.0f;
  const float flo = __int_as_float(0x4B000000 | lo) - 8388608.0f;
  return fmaf(fhi, 65536.0f, flo);
}

// clamp(round_half_even(v / scale), -128, 127) without a divide or a float-to-int convert: the
// quotient from the reciprocal plus one exact-remainder correction, clamped, then rounded by
// adding 1.5 * 2^23 (the add rounds to nearest even) and read back from the bit pattern.
__device__ __forceinline__ int quant_i8_int(float v, float scale, float inv_scale) {
  float q = v * inv_scale;
  const float r = fmaf(-q, scale, v);
  q = fmaf(r, inv_scale, q);
  q = fminf(fmaxf(q, -128.0f), 127.0f);
  return __float_as_int(q + 12582912.0f) - 0x4B400000;
}

__device__ __forceinline__ int8_t quant_i8(float v, float scale) {
  return static_cast<int8_t>(quant_i8_int(v, scale, 1.0f / scale));
}

}  // namespace so101
