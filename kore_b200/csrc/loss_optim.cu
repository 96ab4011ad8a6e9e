// Vocab-wide token log-probability / entropy / cross-entropy gradient and the
// fused AdamW update, for sm_100a.
//
// logprob kernel (one CTA per row, V = 151936 for Qwen3):
//   phase 1: online max / sum-exp / sum z*exp over the row (temperature-scaled)
//            -> lse, logp[target], entropy;
//   phase 2 (optional): overwrite the bf16 logits row with the gradient
//            dz_j = coef_row * inv_temp * (onehot_j - softmax_j).
// The row (300 KB bf16) is re-read from L2 in phase 2. The full [T, V] fp32
// logits tensor is never materialised: callers process token chunks.
// Reference parity: kore/policy/grpo.py:2728-2743 (temperature-scaled
// log-softmax + gather over the full vocabulary in fp32).
//
// AdamW (flat buffers): bf16 params with an optional fp32 master copy; without
// a master the bf16 write uses stochastic rounding (Gupta et al., 2015,
// "Deep Learning with Limited Numerical Precision") driven by a counter-based
// integer hash, so the expected parameter equals the fp32 update. The global
// grad-norm clip factor is read on the device (no host sync).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace {

constexpr int kLpThreads = 512;

KORE_DEV void merge_stats(float& m, float& s, float& w, float m2, float s2, float w2) {
  // combine two partial (max, sum e^{z-max}, sum z e^{z-max}) triples
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; w = w2; return; }
  if (m2 > m) {
    float c = __expf(m - m2);
    s = s * c + s2;
    w = w * c + w2;
    m = m2;
  } else {
    float c = __expf(m2 - m);
    s += s2 * c;
    w += w2 * c;
  }
}

__global__ void __launch_bounds__(kLpThreads) logprob_kernel(
    __nv_bfloat16* __restrict__ logits, int ld, const long* __restrict__ targets, int V,
    float inv_temp, float* __restrict__ logp_out, float* __restrict__ ent_out,
    float* __restrict__ lse_out, const float* __restrict__ coef, int write_grad) {
  const int row = blockIdx.x;
  __nv_bfloat16* z = logits + (size_t)row * ld;
  const int nvec = V / 8;
  float m = -INFINITY, s = 0.f, w = 0.f;
  for (int j = threadIdx.x; j < nvec; j += kLpThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(z + j * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      v[2 * i] = t.x * inv_temp;
      v[2 * i + 1] = t.y * inv_temp;
    }
    float lm = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, v[i]);
    float ls = 0.f, lw = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float e = __expf(v[i] - lm);
      ls += e;
      lw += e * v[i];
    }
    merge_stats(m, s, w, lm, ls, lw);
  }
  // warp then block reduction of the triples
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffff, m, o);
    float s2 = __shfl_xor_sync(0xffffffff, s, o);
    float w2 = __shfl_xor_sync(0xffffffff, w, o);
    merge_stats(m, s, w, m2, s2, w2);
  }
  __shared__ float sm[kLpThreads / 32], ss[kLpThreads / 32], sw[kLpThreads / 32];
  __shared__ float s_lse;
  const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) { sm[wid] = m; ss[wid] = s; sw[wid] = w; }
  __syncthreads();
  if (wid == 0) {
    m = lane < kLpThreads / 32 ? sm[lane] : -INFINITY;
    s = lane < kLpThreads / 32 ? ss[lane] : 0.f;
    w = lane < kLpThreads / 32 ? sw[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float m2 = __shfl_xor_sync(0xffffffff, m, o);
      float s2 = __shfl_xor_sync(0xffffffff, s, o);
      float w2 = __shfl_xor_sync(0xffffffff, w, o);
      merge_stats(m, s, w, m2, s2, w2);
    }
    if (lane == 0) {
      const float lse = m + __logf(s);
      s_lse = lse;
      const long tgt = targets ? targets[row] : -1;
      if (logp_out) {
        float zt = (tgt >= 0 && tgt < V) ? __bfloat162float(z[tgt]) * inv_temp : 0.f;
        logp_out[row] = (tgt >= 0 && tgt < V) ? zt - lse : 0.f;
      }
      if (ent_out) ent_out[row] = lse - w / s;
      if (lse_out) lse_out[row] = lse;
    }
  }
  __syncthreads();
  if (!write_grad) return;
  const float lse = s_lse;
  const float c = coef ? coef[row] * inv_temp : 0.f;
  const long tgt = targets ? targets[row] : -1;
  for (int j = threadIdx.x; j < nvec; j += kLpThreads) {
    uint4 u = *reinterpret_cast<const uint4*>(z + j * 8);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float g[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 t = __bfloat1622float2(h[i]);
      g[2 * i] = -c * __expf(t.x * inv_temp - lse);
      g[2 * i + 1] = -c * __expf(t.y * inv_temp - lse);
    }
    const long base = (long)j * 8;
    if (tgt >= base && tgt < base + 8) g[tgt - base] += c;
    uint4 o;
    o.x = pack_bf16(g[0], g[1]);
    o.y = pack_bf16(g[2], g[3]);
    o.z = pack_bf16(g[4], g[5]);
    o.w = pack_bf16(g[6], g[7]);
    *reinterpret_cast<uint4*>(z + j * 8) = o;
  }
}

// ---------------------------------------------------------------- grad norm
template <typename T>
KORE_DEV float to_f(T v);
template <>
KORE_DEV float to_f<float>(float v) { return v; }
template <>
KORE_DEV float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename G>
__global__ void sumsq_kernel(const G* __restrict__ g, long n, float* __restrict__ out) {
  float acc = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float v = to_f(g[i]);
    acc += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    acc = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
    if (threadIdx.x == 0) atomicAdd(out, acc);
  }
}

// 32-bit integer hash (the "lowbias32" finaliser published by C. Wellons,
// 2018, hash-prospector). Used as a counter-based random source.
KORE_DEV uint32_t hash32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

KORE_DEV __nv_bfloat16 bf16_stochastic(float v, uint32_t rnd) {
  uint32_t b = __float_as_uint(v);
  if ((b & 0x7f800000u) == 0x7f800000u) return __float2bfloat16_rn(v);  // inf/nan
  b += (rnd & 0xffffu);
  b &= 0xffff0000u;
  return __ushort_as_bfloat16((unsigned short)(b >> 16));
}

// p (bf16) [+ master fp32], g (G), m, v fp32. clip factor = min(1, max_norm / (sqrt(sumsq)+1e-6))
template <typename G>
__global__ void adamw_kernel(__nv_bfloat16* __restrict__ p, float* __restrict__ master,
                             const G* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, long n, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, float grad_scale,
                             const float* __restrict__ sumsq, float max_norm, uint32_t seed) {
  float scale = grad_scale;
  if (sumsq != nullptr && max_norm > 0.f) {
    float norm = sqrtf(*sumsq) * grad_scale;
    scale *= fminf(1.f, max_norm / (norm + 1e-6f));
  }
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float gi = to_f(g[i]) * scale;
    float mi = b1 * m[i] + (1.f - b1) * gi;
    float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float w = master ? master[i] : __bfloat162float(p[i]);
    w = w * (1.f - lr * wd);
    w -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    if (master) {
      master[i] = w;
      p[i] = __float2bfloat16_rn(w);
    } else {
      p[i] = bf16_stochastic(w, hash32((uint32_t)i * 0x9E3779B9u ^ seed));
    }
  }
}

// Same update, 8 elements per thread with 16-byte accesses (bf16 grads,
// n % 8 == 0 and 16-byte aligned buffers; checked on the host).
__global__ void adamw_vec8_kernel(__nv_bfloat16* __restrict__ p, float* __restrict__ master,
                                  const __nv_bfloat16* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, long n, float lr, float b1, float b2,
                                  float eps, float wd, float bc1, float bc2, float grad_scale,
                                  const float* __restrict__ sumsq, float max_norm, uint32_t seed) {
  float scale = grad_scale;
  if (sumsq != nullptr && max_norm > 0.f) {
    float norm = sqrtf(*sumsq) * grad_scale;
    scale *= fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const long nv = n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
    const uint4 gu = reinterpret_cast<const uint4*>(g)[i];
    const uint4 pu = reinterpret_cast<const uint4*>(p)[i];
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gu);
    const __nv_bfloat162* ph = reinterpret_cast<const __nv_bfloat162*>(&pu);
    float4* m4 = reinterpret_cast<float4*>(m) + 2 * i;
    float4* v4 = reinterpret_cast<float4*>(v) + 2 * i;
    float4* w4 = master ? reinterpret_cast<float4*>(master) + 2 * i : nullptr;
    float gv[8], mv[8], vv[8], wv[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = __bfloat1622float2(gh[e]);
      gv[2 * e] = a.x * scale;
      gv[2 * e + 1] = a.y * scale;
    }
    {
      const float4 a = m4[0], b = m4[1], c = v4[0], d = v4[1];
      mv[0] = a.x; mv[1] = a.y; mv[2] = a.z; mv[3] = a.w; mv[4] = b.x; mv[5] = b.y; mv[6] = b.z; mv[7] = b.w;
      vv[0] = c.x; vv[1] = c.y; vv[2] = c.z; vv[3] = c.w; vv[4] = d.x; vv[5] = d.y; vv[6] = d.z; vv[7] = d.w;
    }
    if (w4) {
      const float4 a = w4[0], b = w4[1];
      wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w; wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = __bfloat1622float2(ph[e]);
        wv[2 * e] = a.x;
        wv[2 * e + 1] = a.y;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      mv[k] = b1 * mv[k] + (1.f - b1) * gv[k];
      vv[k] = b2 * vv[k] + (1.f - b2) * gv[k] * gv[k];
      wv[k] = wv[k] * (1.f - lr * wd) - lr * (mv[k] / bc1) / (sqrtf(vv[k] / bc2) + eps);
    }
    m4[0] = make_float4(mv[0], mv[1], mv[2], mv[3]);
    m4[1] = make_float4(mv[4], mv[5], mv[6], mv[7]);
    v4[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    v4[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    uint32_t out[4];
    if (w4) {
      w4[0] = make_float4(wv[0], wv[1], wv[2], wv[3]);
      w4[1] = make_float4(wv[4], wv[5], wv[6], wv[7]);
#pragma unroll
      for (int e = 0; e < 4; ++e) out[e] = pack_bf16(wv[2 * e], wv[2 * e + 1]);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat16 lo = bf16_stochastic(wv[2 * e], hash32((uint32_t)(8 * i + 2 * e) * 0x9E3779B9u ^ seed));
        const __nv_bfloat16 hi = bf16_stochastic(wv[2 * e + 1], hash32((uint32_t)(8 * i + 2 * e + 1) * 0x9E3779B9u ^ seed));
        out[e] = (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
      }
    }
    reinterpret_cast<uint4*>(p)[i] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

}  // namespace

// logits: [T, V] bf16 (row stride ld). Returns nothing; fills the given outputs.
void logprob_fwd_bwd(at::Tensor& logits, const c10::optional<at::Tensor>& targets,
                     double inv_temp, const c10::optional<at::Tensor>& logp,
                     const c10::optional<at::Tensor>& entropy, const c10::optional<at::Tensor>& lse,
                     const c10::optional<at::Tensor>& coef, bool write_grad) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1,
              "logits must be bf16 with contiguous rows");
  const int T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0 && logits.stride(0) % 8 == 0, "V and row stride must be multiples of 8");
  if (T == 0) return;
  if (write_grad) TORCH_CHECK(coef.has_value(), "write_grad needs coef");
  c10::cuda::CUDAGuard g(logits.device());
  logprob_kernel<<<T, kLpThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (__nv_bfloat16*)logits.data_ptr(), logits.stride(0),
      targets ? targets->data_ptr<long>() : nullptr, V, (float)inv_temp,
      logp ? logp->data_ptr<float>() : nullptr, entropy ? entropy->data_ptr<float>() : nullptr,
      lse ? lse->data_ptr<float>() : nullptr, coef ? coef->data_ptr<float>() : nullptr,
      write_grad ? 1 : 0);
  check_cuda(cudaGetLastError(), "logprob_fwd_bwd");
}

void sumsq_accumulate(const at::Tensor& g, at::Tensor& out) {
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= 1, "out must be fp32");
  const long n = g.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard gd(g.device());
  int grid = (int)std::min<long>((n + 255) / 256, (long)num_sms(g.get_device()) * 8);
  auto st = at::cuda::getCurrentCUDAStream();
  if (g.scalar_type() == at::kFloat)
    sumsq_kernel<float><<<grid, 256, 0, st>>>(g.data_ptr<float>(), n, out.data_ptr<float>());
  else if (g.scalar_type() == at::kBFloat16)
    sumsq_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)g.data_ptr(), n,
                                                       out.data_ptr<float>());
  else
    TORCH_CHECK(false, "sumsq: unsupported dtype");
  check_cuda(cudaGetLastError(), "sumsq");
}

void adamw_step(at::Tensor& p, const c10::optional<at::Tensor>& master, const at::Tensor& g,
                at::Tensor& m, at::Tensor& v, double lr, double b1, double b2, double eps,
                double wd, int64_t step, double grad_scale, const c10::optional<at::Tensor>& sumsq,
                double max_norm, int64_t seed) {
  TORCH_CHECK(p.scalar_type() == at::kBFloat16 && p.is_contiguous(), "p must be contiguous bf16");
  TORCH_CHECK(m.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat, "m/v must be fp32");
  const long n = p.numel();
  TORCH_CHECK(g.numel() == n && m.numel() == n && v.numel() == n, "adamw: size mismatch");
  if (n == 0) return;
  c10::cuda::CUDAGuard gd(p.device());
  const float bc1 = 1.f - std::pow((float)b1, (float)step);
  const float bc2 = 1.f - std::pow((float)b2, (float)step);
  int grid = (int)std::min<long>((n + 255) / 256, (long)num_sms(p.get_device()) * 8);
  auto st = at::cuda::getCurrentCUDAStream();
  float* mp = master ? master->data_ptr<float>() : nullptr;
  const float* sq = sumsq ? sumsq->data_ptr<float>() : nullptr;
  if (g.scalar_type() == at::kFloat)
    adamw_kernel<float><<<grid, 256, 0, st>>>(
        (__nv_bfloat16*)p.data_ptr(), mp, g.data_ptr<float>(), m.data_ptr<float>(),
        v.data_ptr<float>(), n, lr, b1, b2, eps, wd, bc1, bc2, grad_scale, sq, max_norm,
        (uint32_t)seed);
  else if (n % 8 == 0 && g.is_contiguous() && m.is_contiguous() && v.is_contiguous() &&
           (!master || master->is_contiguous()) &&
           ((reinterpret_cast<uintptr_t>(p.data_ptr()) | reinterpret_cast<uintptr_t>(g.data_ptr()) |
             reinterpret_cast<uintptr_t>(m.data_ptr()) | reinterpret_cast<uintptr_t>(v.data_ptr()) |
             reinterpret_cast<uintptr_t>(mp)) % 16) == 0) {
    const int gv = (int)std::min<long>((n / 8 + 255) / 256, (long)num_sms(p.get_device()) * 8);
    adamw_vec8_kernel<<<gv, 256, 0, st>>>(
        (__nv_bfloat16*)p.data_ptr(), mp, (const __nv_bfloat16*)g.data_ptr(), m.data_ptr<float>(),
        v.data_ptr<float>(), n, lr, b1, b2, eps, wd, bc1, bc2, grad_scale, sq, max_norm, (uint32_t)seed);
  } else
    adamw_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        (__nv_bfloat16*)p.data_ptr(), mp, (const __nv_bfloat16*)g.data_ptr(), m.data_ptr<float>(),
        v.data_ptr<float>(), n, lr, b1, b2, eps, wd, bc1, bc2, grad_scale, sq, max_norm,
        (uint32_t)seed);
  check_cuda(cudaGetLastError(), "adamw");
}

}  // namespace kore
