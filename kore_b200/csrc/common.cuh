// Shared device helpers for the sm_100a kernels of kore_b200.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
//   * mbarrier init / arrive / bounded try_wait (every wait has a time limit and
//     records an error code instead of spinning forever),
//   * TMA tiled loads/stores (cp.async.bulk.tensor; no load uses cluster multicast),
//   * tcgen05 TMEM alloc/dealloc, MMA issue, commit, and TMEM->register loads,
//   * UMMA shared-memory and instruction descriptors.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#define KORE_DEV __device__ __forceinline__

namespace kore {

// Error word of this translation unit (no relocatable device code, so each
// .cu file owns one), read by the host after a launch when checking is enabled.
// Codes: 1 = mbarrier wait timed out, 2 = peer flag wait timed out.
static __device__ int g_error = 0;

// Every translation unit registers a reader for its own error word; the host
// function read_and_clear_device_error() polls all of them.
void register_error_reader(int (*fn)());
static int read_clear_tu_error() {
  int v = 0, z = 0;
  cudaMemcpyFromSymbol(&v, g_error, sizeof(int));
  cudaMemcpyToSymbol(g_error, &z, sizeof(int));
  return v;
}
namespace {
struct TuErrorRegistrar {
  TuErrorRegistrar() { register_error_reader(&read_clear_tu_error); }
};
static TuErrorRegistrar tu_error_registrar_instance;
}  // namespace

// Time limit for any spin-wait inside a kernel (nanoseconds of %globaltimer).
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

KORE_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

KORE_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

KORE_DEV uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

KORE_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n.reg .pred P;\n.reg .b32 R;\n"
      "elect.sync R|P, 0xffffffff;\n"
      "selp.b32 %0, 1, 0, P;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
KORE_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
KORE_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
KORE_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n.reg .b64 st;\nmbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
               : "memory");
}
KORE_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n.reg .b64 st;\nmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
KORE_DEV bool mbar_try_wait(uint32_t bar_addr, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred P;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n"
      "selp.b32 %0, 1, 0, P;\n}\n"
      : "=r"(ok)
      : "r"(bar_addr), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and records error code 1) if the phase did not
// complete within kWaitTimeoutNs. Callers abandon their loop on false.
KORE_DEV bool mbar_wait(uint64_t* bar, uint32_t phase) {
  uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, phase)) return true;
  uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(a, phase)) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicExch(&g_error, 1);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
KORE_DEV void tma_prefetch_desc(const CUtensorMap* d) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(d)) : "memory");
}
KORE_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* d, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(d)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
KORE_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* d, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(d)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
KORE_DEV void tma_store_2d(const CUtensorMap* d, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(d)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
// Element-wise atomic add of a shared-memory box into global memory (TMA reduce).
KORE_DEV void tma_reduce_add_3d(const CUtensorMap* d, const void* smem_src, int x, int y, int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(d)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
KORE_DEV void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
KORE_DEV void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
KORE_DEV void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
KORE_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Order this thread's generic-proxy global accesses with later async-proxy (TMA) ones.
KORE_DEV void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
KORE_DEV void st_release_gpu_s32(int* a, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
KORE_DEV int ld_acquire_gpu_s32(const int* a) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
// Bounded wait until *flag >= want (error code 4 after kWaitTimeoutNs).
KORE_DEV bool wait_flag_ge(const int* flag, int want) {
  if (ld_acquire_gpu_s32(flag) >= want) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    __nanosleep(64);
    if (ld_acquire_gpu_s32(flag) >= want) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      atomicExch(&g_error, 4);
      return false;
    }
  }
}

// ---------------------------------------------------------------- tcgen05
// Allocate `ncols` TMEM columns (power of two >= 32); whole warp must call.
KORE_DEV void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
KORE_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
KORE_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KORE_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, bf16/f16 inputs, fp32 accumulate.
KORE_DEV void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Same with the A operand read from TMEM (the "TS" form).
KORE_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Make the mbarrier track completion of all previously issued MMAs of this thread.
KORE_DEV void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Each thread of the warp reads 32 consecutive 32-bit columns of its TMEM lane.
KORE_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
KORE_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
KORE_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]));
}
KORE_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
KORE_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor for a 128-byte-swizzled tile (the layout TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B). Byte offsets are encoded >> 4.
//   K-major : rows of 128 B (64 bf16 along K), 8-row groups `sbo` bytes apart.
//   MN-major: 128 B runs along M/N, 64-element MN blocks `lbo` bytes apart,
//             8-row K groups `sbo` bytes apart.
KORE_DEV uint64_t make_sw128_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, shape MxN, operand majors.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                         // D format f32
         | (1u << 7)                       // A bf16
         | (1u << 10)                      // B bf16
         | ((a_mn ? 1u : 0u) << 15)        // A major
         | ((b_mn ? 1u : 0u) << 16)        // B major
         | ((uint32_t)(N >> 3) << 17)      // N / 8
         | ((uint32_t)(M >> 4) << 24);     // M / 16
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A 2-CTA cluster shares one UMMA: the leader (rank 0) issues 256-row MMAs
// whose A rows and B columns are split over the two CTAs' shared memory, and
// each CTA's TMEM receives its 128 rows of the accumulator. Plain (non-multicast)
// TMA loads from each CTA signal the leader's barrier; completion of the MMAs
// is broadcast to both CTAs' barriers by tcgen05.commit with a CTA mask.
KORE_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
KORE_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
KORE_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (address from mapa_shared).
KORE_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on
// the mbarrier at `bar_cluster_addr`, which may be in the peer CTA of the pair.
KORE_DEV void tma_load_2d_pair(void* smem_dst, const CUtensorMap* d, uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(d)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
KORE_DEV void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
KORE_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
KORE_DEV void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                               uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive (once) on the mbarrier at the same offset in every CTA of `cta_mask`
// when all previously issued pair MMAs of this thread have completed.
KORE_DEV void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)), "h"(cta_mask)
      : "memory");
}

KORE_DEV uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Packed fp32 pairs (sm_100a f32x2 instructions): one issue slot for two lanes' worth.
KORE_DEV uint64_t f2_pack(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
KORE_DEV void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
KORE_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
KORE_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
KORE_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
KORE_DEV float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

}  // namespace kore
