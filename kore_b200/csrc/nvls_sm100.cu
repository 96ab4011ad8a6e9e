// NVLink SHARP (NVLS) data plane: the sharded optimizer step with the
// gradient reduction done inside the NVSwitch and the parameter all-gather
// done as one multicast store.
//
// Gradients and parameters live in buffers bound to an NVLink multicast
// object (one physical copy per GPU, one multicast address for all). For its
// own shard, a rank
//   1. reads the sum over all ranks of the bf16 gradients with
//      multimem.ld_reduce (the switch adds the W copies, fp32 accumulation,
//      one bf16 result per element),
//   2. applies clipped AdamW to its fp32 shard state,
//   3. stores the new bf16 parameters with multimem.st, which writes them into
//      every rank's parameter buffer at once.
// Each gradient byte crosses NVLink once (into the switch) and each parameter
// byte once (out of it), instead of W-1 times each for peer loads / stores.
//
// A second kernel computes the global sum of squares of the reduced gradient
// (for clipping) from the same multicast reads. Ordering across ranks (all
// gradients written before the reads; all parameter stores visible before the
// next forward) is the caller's: the flag barrier of the symmetric heap,
// bounded like every wait in this package. Nothing here waits.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace nvls {

KORE_DEV void ld_reduce_bf16x8(const void* mc, uint32_t (&r)[4]) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(reinterpret_cast<uint64_t>(mc))
               : "memory");
}

KORE_DEV void st_multicast_16b(void* mc, const uint32_t (&r)[4]) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(reinterpret_cast<uint64_t>(mc)),
               "f"(__uint_as_float(r[0])), "f"(__uint_as_float(r[1])), "f"(__uint_as_float(r[2])),
               "f"(__uint_as_float(r[3]))
               : "memory");
}

KORE_DEV void bf16x8_to_f32(const uint32_t (&r)[4], float (&f)[8]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&r[e]);
    float2 t = __bfloat1622float2(h);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

// The same bytes are reached through the multicast and the unicast mapping:
// order accesses across the two virtual aliases.
KORE_DEV void fence_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

KORE_DEV uint32_t mix32(uint32_t x) {       // integer hash for stochastic rounding
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// out[0] += sum over this rank's shard of (reduced gradient * gscale)^2
__global__ void sumsq_kernel(const __nv_bfloat16* mc_grad, long n, float gscale, float* out) {
  fence_alias();
  float acc = 0.f;
  const long nvec = n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    uint32_t r[4];
    float f[8];
    ld_reduce_bf16x8(mc_grad + i * 8, r);
    bf16x8_to_f32(r, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += (f[k] * gscale) * (f[k] * gscale);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += red[w];
    atomicAdd(out, t);
  }
}

// AdamW on this rank's shard; mc_grad / mc_param point at the shard's first
// element in the multicast mapping; own_param at the same element in this
// rank's own (unicast) copy.
__global__ void adamw_kernel(const __nv_bfloat16* mc_grad, __nv_bfloat16* mc_param,
                             const __nv_bfloat16* own_param, float* __restrict__ master, float* __restrict__ m,
                             float* __restrict__ v, long n, long elem0, float gscale, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, const float* __restrict__ sumsq,
                             float max_norm, uint32_t seed) {
  fence_alias();
  float clip = 1.f;
  if (sumsq != nullptr && max_norm > 0.f) clip = fminf(1.f, max_norm / (sqrtf(*sumsq) + 1e-6f));
  const long nvec = n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    uint32_t r[4];
    float g[8], w[8];
    ld_reduce_bf16x8(mc_grad + i * 8, r);
    bf16x8_to_f32(r, g);
    if (master != nullptr) {
      const float4 a = reinterpret_cast<const float4*>(master + i * 8)[0];
      const float4 b = reinterpret_cast<const float4*>(master + i * 8)[1];
      w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    } else {
      const uint4 cur = *reinterpret_cast<const uint4*>(own_param + i * 8);
      const uint32_t c[4] = {cur.x, cur.y, cur.z, cur.w};
      bf16x8_to_f32(c, w);
    }
    float4* m4 = reinterpret_cast<float4*>(m + i * 8);
    float4* v4 = reinterpret_cast<float4*>(v + i * 8);
    const float4 ma = m4[0], mb = m4[1], va = v4[0], vb = v4[1];
    float mv[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
    float vv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float gi = g[k] * gscale * clip;
      mv[k] = b1 * mv[k] + (1.f - b1) * gi;
      vv[k] = b2 * vv[k] + (1.f - b2) * gi * gi;
      w[k] = w[k] * (1.f - lr * wd) - lr * (mv[k] / bc1) / (sqrtf(vv[k] / bc2) + eps);
    }
    m4[0] = make_float4(mv[0], mv[1], mv[2], mv[3]);
    m4[1] = make_float4(mv[4], mv[5], mv[6], mv[7]);
    v4[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    v4[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    if (master != nullptr) {
      reinterpret_cast<float4*>(master + i * 8)[0] = make_float4(w[0], w[1], w[2], w[3]);
      reinterpret_cast<float4*>(master + i * 8)[1] = make_float4(w[4], w[5], w[6], w[7]);
    }
    uint32_t out[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float a = w[2 * e], b = w[2 * e + 1];
      if (master == nullptr) {                   // stochastic rounding of the bf16 parameters
        const uint32_t j = (uint32_t)(elem0 + i * 8 + 2 * e);
        uint32_t ua = __float_as_uint(a) + (mix32(j * 0x9E3779B9u ^ seed) & 0xffffu);
        uint32_t ub = __float_as_uint(b) + (mix32((j + 1) * 0x9E3779B9u ^ seed) & 0xffffu);
        a = __uint_as_float(ua & 0xffff0000u);
        b = __uint_as_float(ub & 0xffff0000u);
      }
      out[e] = pack_bf16(a, b);
    }
    st_multicast_16b(mc_param + i * 8, out);
  }
  fence_alias();
  __threadfence_system();                      // the multicast stores precede the caller's barrier
}

inline int grid_for(long nvec) {
  return (int)std::min<long>(std::max<long>(1, (nvec + 255) / 256), 148L * 8);
}

}  // namespace nvls

// Host entry points. Pointers are raw device addresses (the multicast base of
// the symmetric buffers plus an element offset), n a multiple of 8, offsets
// 16-byte aligned.
void nvls_sumsq(int64_t mc_grad, int64_t n, double gscale, at::Tensor& out) {
  TORCH_CHECK(n % 8 == 0 && mc_grad % 16 == 0, "nvls sumsq: n % 8 and 16-byte alignment");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat, "nvls sumsq: out fp32 CUDA");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(out.device());
  nvls::sumsq_kernel<<<nvls::grid_for(n / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(mc_grad), n, (float)gscale, out.data_ptr<float>());
  check_cuda(cudaGetLastError(), "nvls sumsq");
}

void nvls_adamw(int64_t mc_grad, int64_t mc_param, const at::Tensor& own_param,
                const c10::optional<at::Tensor>& master, at::Tensor& m, at::Tensor& v, int64_t elem0, double gscale,
                double lr, double b1, double b2, double eps, double wd, int64_t step,
                const c10::optional<at::Tensor>& sumsq, double max_norm, int64_t seed) {
  const long n = m.numel();
  TORCH_CHECK(n % 8 == 0 && mc_grad % 16 == 0 && mc_param % 16 == 0, "nvls adamw: n % 8 and 16-byte alignment");
  TORCH_CHECK(v.numel() == n && own_param.numel() == n && m.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat && own_param.scalar_type() == at::kBFloat16,
              "nvls adamw: shapes / dtypes");
  TORCH_CHECK(!master || (master->numel() == n && master->scalar_type() == at::kFloat), "nvls adamw: master");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(m.device());
  const float bc1 = 1.f - (float)std::pow(b1, (double)step), bc2 = 1.f - (float)std::pow(b2, (double)step);
  nvls::adamw_kernel<<<nvls::grid_for(n / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(mc_grad), reinterpret_cast<__nv_bfloat16*>(mc_param),
      reinterpret_cast<const __nv_bfloat16*>(own_param.data_ptr()), master ? master->data_ptr<float>() : nullptr,
      m.data_ptr<float>(), v.data_ptr<float>(), n, elem0, (float)gscale, (float)lr, (float)b1, (float)b2,
      (float)eps, (float)wd, bc1, bc2, sumsq ? sumsq->data_ptr<float>() : nullptr, (float)max_norm,
      (uint32_t)seed);
  check_cuda(cudaGetLastError(), "nvls adamw");
}

}  // namespace kore
