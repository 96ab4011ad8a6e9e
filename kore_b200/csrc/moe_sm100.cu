// Mixture-of-experts kernels for sm_100a (Qwen3-MoE: 128 experts, top-8).
//   * moe_route_fwd: softmax over experts, top-k selection by k rounds of a
//                    warp argmax, optional renormalisation of the k weights
//   * moe_route_bwd: gradient of the router logits from d(weights)
//   * moe_combine:   y[t] = sum_j w[t,j] * src[pos[t,j]] (+ residual); with
//                    w == nullptr it is the un-permute sum used by the backward
//   * moe_combine_bwd: dsrc[pos[t,j]] = w[t,j] * dy[t];  dw[t,j] = <dy[t], src[pos[t,j]]>
// The expert GEMMs run on the grouped tcgen05 GEMM; the row permutation is a
// gather with the embedding kernel. Reference parity: HF Qwen3MoeSparseMoeBlock
// (router softmax -> top-k -> norm_topk_prob -> experts -> weighted sum); the
// reference only has MoE as task content (kore/tasks/fused_moe_silu_bf16).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace moe {

constexpr int kMaxE = 256;
constexpr int kMaxK = 16;

// one warp per token; E <= 256 (E / 32 values per lane)
__global__ void route_fwd_kernel(const float* __restrict__ logits, int T, int E, int k, int norm,
                                 float* __restrict__ probs, int* __restrict__ idx, float* __restrict__ w) {
  const long tok = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (tok >= T) return;
  const int per = (E + 31) / 32;
  float v[kMaxE / 32];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxE / 32; ++i) {
    const int e = lane + 32 * i;
    v[i] = (i < per && e < E) ? logits[tok * E + e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxE / 32; ++i) {
    v[i] = (v[i] == -INFINITY) ? 0.f : __expf(v[i] - mx);
    sum += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffff, sum, o);
  const float inv = 1.f / sum;
#pragma unroll
  for (int i = 0; i < kMaxE / 32; ++i) {
    v[i] *= inv;
    const int e = lane + 32 * i;
    if (i < per && e < E) probs[tok * E + e] = v[i];
  }
  float sel[kMaxK];
  int sid[kMaxK];
  float tot = 0.f;
  for (int j = 0; j < k; ++j) {
    float best = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
      const int e = lane + 32 * i;
      if (i < per && e < E && (v[i] > best || (v[i] == best && e < bi))) { best = v[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float b2 = __shfl_xor_sync(0xffffffff, best, o);
      const int i2 = __shfl_xor_sync(0xffffffff, bi, o);
      if (b2 > best || (b2 == best && i2 < bi)) { best = b2; bi = i2; }
    }
    sel[j] = best;
    sid[j] = bi;
    tot += best;
    // remove the winner from further rounds
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i)
      if (lane + 32 * i == bi) v[i] = -2.f;
  }
  if (lane == 0) {
    for (int j = 0; j < k; ++j) {
      idx[tok * k + j] = sid[j];
      w[tok * k + j] = norm ? sel[j] / tot : sel[j];
    }
  }
}

// dz = p * (ds - <p, ds>), with ds scattered from the selected entries:
// norm:    ds_j = (g_j - sum_l g_l w_l) / S,  S = sum of selected probs
// no norm: ds_j = g_j
__global__ void route_bwd_kernel(const float* __restrict__ probs, const int* __restrict__ idx,
                                 const float* __restrict__ w, const float* __restrict__ dw, int T, int E,
                                 int k, int norm, float* __restrict__ dlogits) {
  const long tok = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (tok >= T) return;
  float S = 0.f, gw = 0.f;
  for (int j = 0; j < k; ++j) {
    S += probs[tok * E + idx[tok * k + j]];
    gw += dw[tok * k + j] * w[tok * k + j];
  }
  float dot = 0.f;  // <p, ds>
  for (int j = 0; j < k; ++j) {
    const float ds = norm ? (dw[tok * k + j] - gw) / S : dw[tok * k + j];
    dot += probs[tok * E + idx[tok * k + j]] * ds;
  }
  for (int e = lane; e < E; e += 32) {
    float ds = 0.f;
    for (int j = 0; j < k; ++j)
      if (idx[tok * k + j] == e) ds = norm ? (dw[tok * k + j] - gw) / S : dw[tok * k + j];
    dlogits[tok * E + e] = probs[tok * E + e] * (ds - dot);
  }
}

// one warp per token row; H multiple of 256 handled in 8-element chunks
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ pos,
                               const float* __restrict__ w, const __nv_bfloat16* __restrict__ resid,
                               __nv_bfloat16* __restrict__ out, int T, int H, int k) {
  const long tok = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (tok >= T) return;
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (resid) {
      const uint4 u = *reinterpret_cast<const uint4*>(resid + tok * H + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] = f.x;
        acc[2 * e + 1] = f.y;
      }
    }
    for (int j = 0; j < k; ++j) {
      const int p = pos[tok * k + j];
      if (p < 0) continue;
      const float ww = w ? w[tok * k + j] : 1.f;
      const uint4 u = *reinterpret_cast<const uint4*>(src + (long)p * H + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += ww * f.x;
        acc[2 * e + 1] += ww * f.y;
      }
    }
    *reinterpret_cast<uint4*>(out + tok * H + c) =
        make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                   pack_bf16(acc[6], acc[7]));
  }
}

// one warp per (token, slot)
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ src,
                                   const int* __restrict__ pos, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ dsrc, float* __restrict__ dw, int T, int H,
                                   int k) {
  const long pair = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (pair >= (long)T * k) return;
  const long tok = pair / k;
  const int p = pos[pair];
  if (p < 0) {
    if (lane == 0) dw[pair] = 0.f;
    return;
  }
  const float ww = w[pair];
  float dot = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 gu = *reinterpret_cast<const uint4*>(dy + tok * H + c);
    const uint4 su = *reinterpret_cast<const uint4*>(src + (long)p * H + c);
    const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&gu);
    const __nv_bfloat162* s = reinterpret_cast<const __nv_bfloat162*>(&su);
    float o[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 gf = __bfloat1622float2(g[e]);
      float2 sf = __bfloat1622float2(s[e]);
      dot += gf.x * sf.x + gf.y * sf.y;
      o[2 * e] = ww * gf.x;
      o[2 * e + 1] = ww * gf.y;
    }
    *reinterpret_cast<uint4*>(dsrc + (long)p * H + c) =
        make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffff, dot, o);
  if (lane == 0) dw[pair] = dot;
}

inline int warps_grid(long n, int warps_per_block = 8) {
  return (int)((n + warps_per_block - 1) / warps_per_block);
}

}  // namespace moe

void moe_route_fwd(const at::Tensor& logits, int64_t k, bool norm, at::Tensor& probs, at::Tensor& idx,
                   at::Tensor& w) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "logits fp32 contiguous [T,E]");
  const int T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E <= moe::kMaxE && k <= moe::kMaxK && k <= E, "E <= 256 and k <= 16");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  moe::route_fwd_kernel<<<moe::warps_grid(T), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      logits.data_ptr<float>(), T, E, k, norm ? 1 : 0, probs.data_ptr<float>(), idx.data_ptr<int>(),
      w.data_ptr<float>());
  check_cuda(cudaGetLastError(), "moe_route_fwd");
}

void moe_route_bwd(const at::Tensor& probs, const at::Tensor& idx, const at::Tensor& w, const at::Tensor& dw,
                   bool norm, at::Tensor& dlogits) {
  const int T = probs.size(0), E = probs.size(1), k = idx.size(1);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(probs.device());
  moe::route_bwd_kernel<<<moe::warps_grid(T), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      probs.data_ptr<float>(), idx.data_ptr<int>(), w.data_ptr<float>(), dw.data_ptr<float>(), T, E, k,
      norm ? 1 : 0, dlogits.data_ptr<float>());
  check_cuda(cudaGetLastError(), "moe_route_bwd");
}

void moe_combine(const at::Tensor& src, const at::Tensor& pos, const c10::optional<at::Tensor>& w,
                 const c10::optional<at::Tensor>& resid, at::Tensor& out) {
  const int T = pos.size(0), k = pos.size(1), H = src.size(1);
  TORCH_CHECK(H % 8 == 0 && src.is_contiguous() && out.is_contiguous(), "combine: contiguous rows, H % 8");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  moe::combine_kernel<<<moe::warps_grid(T), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)src.data_ptr(), pos.data_ptr<int>(), w ? w->data_ptr<float>() : nullptr,
      resid ? (const __nv_bfloat16*)resid->data_ptr() : nullptr, (__nv_bfloat16*)out.data_ptr(), T, H, k);
  check_cuda(cudaGetLastError(), "moe_combine");
}

void moe_combine_bwd(const at::Tensor& dy, const at::Tensor& src, const at::Tensor& pos, const at::Tensor& w,
                     at::Tensor& dsrc, at::Tensor& dw) {
  const int T = pos.size(0), k = pos.size(1), H = src.size(1);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  moe::combine_bwd_kernel<<<moe::warps_grid((long)T * k), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)src.data_ptr(), pos.data_ptr<int>(),
      w.data_ptr<float>(), (__nv_bfloat16*)dsrc.data_ptr(), dw.data_ptr<float>(), T, H, k);
  check_cuda(cudaGetLastError(), "moe_combine_bwd");
}

}  // namespace kore
