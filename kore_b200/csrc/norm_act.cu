// Memory-bound fused kernels of the Qwen3 decoder for sm_100a:
//   * RMSNorm forward / backward (+ fused residual-gradient add, dW reduction)
//   * per-head q_norm/k_norm RMSNorm fused with rotary embedding, fwd / bwd
//   * SwiGLU (silu(gate) * up) forward / backward
//   * token embedding gather / gradient scatter-add
// All math is fp32 in registers; bf16 in HBM; 16-byte vector accesses.
//
// Reference parity: HF Qwen3RMSNorm / apply_rotary_pos_emb / SiLU-gated MLP
// as used by the reference's trainers (kore/policy/configs.py:550-567 picks the
// Qwen3 decoder layer; the math itself lives in transformers).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma_host.h"

namespace kore {

namespace {

KORE_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

template <int NT>
KORE_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) t += red[i];
  return t;
}

KORE_DEV void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
KORE_DEV void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

constexpr int kNormThreads = 128;
constexpr int kMaxVecPerThread = 8;  // H <= 128 * 8 * 8 = 8192

// ---------------------------------------------------------------- RMSNorm fwd
// THREADS x VPT 8-element vectors cover a row (H <= THREADS * VPT * 8); the
// template keeps the per-thread arrays exactly as large as the row needs.
template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS) rmsnorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int rows, int H, float eps) {
  __shared__ float red[THREADS / 32];
  const int nvec = H / 8;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* xr = x + (size_t)r * H;
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int j = threadIdx.x + i * THREADS;
      if (j < nvec) {
        load8(xr + j * 8, v[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
      }
    }
    ss = block_sum<THREADS>(ss, red);
    const float rs = rsqrtf(ss / H + eps);
    if (rstd_out && threadIdx.x == 0) rstd_out[r] = rs;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int j = threadIdx.x + i * THREADS;
      if (j < nvec) {
        float wv[8];
        load8(w + j * 8, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = v[i][e] * rs * wv[e];
        store8(y + (size_t)r * H + j * 8, v[i]);
      }
    }
  }
}

// ---------------------------------------------------------------- RMSNorm bwd
// dx = rstd * (w*dy - xhat * mean(xhat*w*dy)) (+ dres);  dw += sum_rows dy*xhat
// Persistent blocks walk rows with a stride of the grid. Each thread keeps the
// raw bf16 vectors of its columns (x, dy, dres) and loads the NEXT row's
// vectors before it reduces the current one, so two rows' loads are in
// flight per thread across the block-wide reduction; dw accumulates in
// registers and is added once per block at the end.
KORE_DEV void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int THREADS, int VPT>
__global__ void __launch_bounds__(THREADS) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
    const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
    float* __restrict__ dw, int rows, int H) {
  __shared__ float red[THREADS / 32];
  const int nvec = H / 8;
  float dwacc[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) dwacc[i][e] = 0.f;
  uint4 cx[VPT], cg[VPT], cr[VPT];
  auto load_row = [&](int r, uint4 (&px)[VPT], uint4 (&pg)[VPT], uint4 (&pr)[VPT]) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = threadIdx.x + i * THREADS;
      if (j < nvec) {
        px[i] = __ldg(reinterpret_cast<const uint4*>(x + (size_t)r * H + j * 8));
        pg[i] = __ldg(reinterpret_cast<const uint4*>(dy + (size_t)r * H + j * 8));
        if (dres) pr[i] = __ldg(reinterpret_cast<const uint4*>(dres + (size_t)r * H + j * 8));
      }
    }
  };
  int r = blockIdx.x;
  if (r < rows) load_row(r, cx, cg, cr);
  for (; r < rows; r += gridDim.x) {
    uint4 nx[VPT], ng[VPT], nr[VPT];
    const int rn = r + gridDim.x;
    if (rn < rows) load_row(rn, nx, ng, nr);
    const float rs = rstd[r];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = threadIdx.x + i * THREADS;
      if (j < nvec) {
        float xv[8], g[8], wv[8];
        unpack8(cx[i], xv);
        unpack8(cg[i], g);
        load8(w + j * 8, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float xh = xv[e] * rs;
          dwacc[i][e] += g[e] * xh;
          dot += g[e] * wv[e] * xh;
        }
      }
    }
    dot = block_sum<THREADS>(dot, red) / H;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int j = threadIdx.x + i * THREADS;
      if (j < nvec) {
        float xv[8], g[8], wv[8], o[8];
        unpack8(cx[i], xv);
        unpack8(cg[i], g);
        load8(w + j * 8, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rs * (g[e] * wv[e] - xv[e] * rs * dot);
        if (dres) {
          float d[8];
          unpack8(cr[i], d);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] += d[e];
        }
        store8(dx + (size_t)r * H + j * 8, o);
      }
    }
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      cx[i] = nx[i];
      cg[i] = ng[i];
      cr[i] = nr[i];
    }
  }
  if (dw) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      int j = threadIdx.x + i * THREADS;
      if (j < nvec)
#pragma unroll
        for (int e = 0; e < 8; ++e) atomicAdd(dw + j * 8 + e, dwacc[i][e]);
    }
  }
}

// ------------------------------------------- q/k per-head RMSNorm + RoPE (fwd)
// qkv: [T, (Hq + 2*Hkv) * D] raw projections. out: [T, (Hq + Hkv) * D] normed+rotated q,k.
// One 256-thread block per token; warp w handles heads w, w + 8, ... (up to
// kQkMaxHeadsPerWarp each), D == 128 (4 elements per lane; lane l pairs with
// l^16 for rotate-half). The token's position and its cos/sin row are read
// once per warp, and all of a warp's head loads are issued before the first
// reduction, so a warp keeps several rows in flight.
// cos/sin tables: [max_pos, D/2] fp32.
constexpr int kQkMaxHeadsPerWarp = 12;   // Hq + Hkv <= 96

__global__ void __launch_bounds__(256) qk_norm_rope_fwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qw,
    const __nv_bfloat16* __restrict__ kw, const int* __restrict__ pos, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, __nv_bfloat16* __restrict__ out, float* __restrict__ rstd, int T,
    int Hq, int Hkv, float eps) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int heads = Hq + Hkv;
  const int t = blockIdx.x;
  if (t >= T) return;
  const int in_stride = (Hq + 2 * Hkv) * D;
  const __nv_bfloat16* src = qkv + (size_t)t * in_stride + lane * 4;
  uint2 raw[kQkMaxHeadsPerWarp];
#pragma unroll
  for (int i = 0; i < kQkMaxHeadsPerWarp; ++i) {
    const int h = warp + 8 * i;
    if (h < heads) raw[i] = __ldg(reinterpret_cast<const uint2*>(src + h * D));
  }
  const int p = pos[t];
  const int fi = (lane & 15) * 4;
  const float4 c4 = __ldg(reinterpret_cast<const float4*>(cos_t + (size_t)p * (D / 2) + fi));
  const float4 s4 = __ldg(reinterpret_cast<const float4*>(sin_t + (size_t)p * (D / 2) + fi));
  const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
  float wq[4], wk[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    wq[e] = __bfloat162float(qw[lane * 4 + e]);
    wk[e] = __bfloat162float(kw[lane * 4 + e]);
  }
#pragma unroll
  for (int i = 0; i < kQkMaxHeadsPerWarp; ++i) {
    const int h = warp + 8 * i;
    if (h >= heads) break;
    float v[4];
    {
      float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&raw[i].x));
      float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&raw[i].y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    }
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / D + eps);
    if (rstd && lane == 0) rstd[(size_t)t * heads + h] = rs;
    const bool is_q = h < Hq;
    float n[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) n[e] = v[e] * rs * (is_q ? wq[e] : wk[e]);
    // rotate_half: x1 = n[:64], x2 = n[64:]; out1 = x1*c - x2*s; out2 = x2*c + x1*s
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float partner = __shfl_xor_sync(0xffffffff, n[e], 16);
      o[e] = lane < 16 ? n[e] * cs[e] - partner * sn[e] : n[e] * cs[e] + partner * sn[e];
    }
    uint2 u;
    u.x = pack_bf16(o[0], o[1]);
    u.y = pack_bf16(o[2], o[3]);
    *reinterpret_cast<uint2*>(out + (size_t)t * heads * D + h * D + lane * 4) = u;
  }
}

// --------------------------------------------------- q/k norm + RoPE (bwd)
// dout: [T, (Hq+Hkv)*D] grads of the rotated q,k. Writes dqkv[:, :(Hq+Hkv)*D]
// (row stride (Hq+2Hkv)*D) and accumulates dqw/dkw (fp32, [D]).
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dout,
                                        const __nv_bfloat16* __restrict__ qkv,
                                        const __nv_bfloat16* __restrict__ qw,
                                        const __nv_bfloat16* __restrict__ kw,
                                        const int* __restrict__ pos, const float* __restrict__ cos_t,
                                        const float* __restrict__ sin_t,
                                        __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dqw,
                                        float* __restrict__ dkw, int T, int Hq, int Hkv,
                                        float eps) {
  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  const int heads = Hq + Hkv;
  const int in_stride = (Hq + 2 * Hkv) * D;
  float accq[4] = {0, 0, 0, 0}, acck[4] = {0, 0, 0, 0};
  const long nwarps_total = (long)gridDim.x * (blockDim.x / 32);
  for (long gw = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; gw < (long)T * heads;
       gw += nwarps_total) {
    const int t = gw / heads, h = gw % heads;
    float g[4], v[4];
    {
      uint2 u = *reinterpret_cast<const uint2*>(dout + (size_t)t * heads * D + h * D + lane * 4);
      float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
      float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
      g[0] = a.x; g[1] = a.y; g[2] = b.x; g[3] = b.y;
      uint2 w2 = *reinterpret_cast<const uint2*>(qkv + (size_t)t * in_stride + h * D + lane * 4);
      a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w2.x));
      b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w2.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    }
    // inverse rotation of the gradient: dn1 = g1*c + g2*s ; dn2 = g2*c - g1*s
    float gp[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) gp[e] = __shfl_xor_sync(0xffffffff, g[e], 16);
    const int p = pos[t];
    const int fi = (lane & 15) * 4;
    float dn[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float c = cos_t[(size_t)p * (D / 2) + fi + e];
      float s = sin_t[(size_t)p * (D / 2) + fi + e];
      dn[e] = lane < 16 ? g[e] * c + gp[e] * s : g[e] * c - gp[e] * s;
    }
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / D + eps);
    const __nv_bfloat16* wt = (h < Hq ? qw : kw) + lane * 4;
    float gw_[4], xh[4], dot = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      xh[e] = v[e] * rs;
      float wv = __bfloat162float(wt[e]);
      if (h < Hq) accq[e] += dn[e] * xh[e]; else acck[e] += dn[e] * xh[e];
      gw_[e] = dn[e] * wv;
      dot += gw_[e] * xh[e];
    }
    dot = warp_sum(dot) / D;
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = rs * (gw_[e] - xh[e] * dot);
    uint2 u;
    u.x = pack_bf16(o[0], o[1]);
    u.y = pack_bf16(o[2], o[3]);
    *reinterpret_cast<uint2*>(dqkv + (size_t)t * in_stride + h * D + lane * 4) = u;
  }
  // reduce weight grads within the block, then one atomic per element
  __shared__ float sq[8][128], sk[8][128];
  const int w = threadIdx.x / 32;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    sq[w][lane * 4 + e] = accq[e];
    sk[w][lane * 4 + e] = acck[e];
  }
  __syncthreads();
  if (threadIdx.x < 128) {
    float a = 0.f, b = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) {
      a += sq[i][threadIdx.x];
      b += sk[i][threadIdx.x];
    }
    atomicAdd(dqw + threadIdx.x, a);
    atomicAdd(dkw + threadIdx.x, b);
  }
}

// ---------------------------------------------------------------- SwiGLU
// gu: [T, 2F] = [gate | up]; out[T, F] = silu(gate) * up
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ out,
                                  long T, int F, int ld_in) {
  const long nvec = T * (F / 8);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    const long t = i / (F / 8);
    const int j = (i % (F / 8)) * 8;
    float g[8], u[8], o[8];
    load8(gu + t * ld_in + j, g);
    load8(gu + t * ld_in + F + j, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = g[e] / (1.f + __expf(-g[e])) * u[e];
    store8(out + t * F + j, o);
  }
}

// dgu[:, :F] = dout * up * dsilu(gate); dgu[:, F:] = dout * silu(gate). dgu may alias gu.
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* gu,
                                  __nv_bfloat16* dgu, long T, int F, int ld) {
  const long nvec = T * (F / 8);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    const long t = i / (F / 8);
    const int j = (i % (F / 8)) * 8;
    float g[8], u[8], d[8], dg[8], du[8];
    load8(gu + t * ld + j, g);
    load8(gu + t * ld + F + j, u);
    load8(dout + t * F + j, d);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float s = 1.f / (1.f + __expf(-g[e]));
      float si = g[e] * s;
      du[e] = d[e] * si;
      dg[e] = d[e] * u[e] * (s + si * (1.f - s));
    }
    store8(dgu + t * ld + j, dg);
    store8(dgu + t * ld + F + j, du);
  }
}

// ---------------------------------------------------------------- embedding
__global__ void embed_fwd_kernel(const long* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, long T, int H) {
  const int nvec = H / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < T * nvec; i += (long)gridDim.x * blockDim.x) {
    const long t = i / nvec;
    const int j = (i % nvec) * 8;
    *reinterpret_cast<uint4*>(out + t * H + j) =
        *reinterpret_cast<const uint4*>(table + ids[t] * (long)H + j);
  }
}
KORE_DEV void atomic_add8(float* dst, const float (&g)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) atomicAdd(dst + e, g[e]);
}
KORE_DEV void atomic_add8(__nv_bfloat16* dst, const float (&g)[8]) {
  __nv_bfloat162* d2 = reinterpret_cast<__nv_bfloat162*>(dst);
#pragma unroll
  for (int e = 0; e < 4; ++e) atomicAdd(d2 + e, __floats2bfloat162_rn(g[2 * e], g[2 * e + 1]));
}
template <typename G>
__global__ void embed_bwd_kernel(const long* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                 G* __restrict__ dtable, long T, int H) {
  const int nvec = H / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < T * nvec; i += (long)gridDim.x * blockDim.x) {
    const long t = i / nvec;
    const int j = (i % nvec) * 8;
    float g[8];
    load8(dy + t * H + j, g);
    atomic_add8(dtable + ids[t] * (long)H + j, g);
  }
}

int grid_for(long work, int threads, int dev) {
  long b = (work + threads - 1) / threads;
  long cap = (long)num_sms(dev) * 16;
  return (int)std::max<long>(1, std::min(b, cap));
}

void check_bf16_2d(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.is_contiguous(), name,
              " must be a contiguous CUDA bf16 tensor");
}

}  // namespace

// ============================================================== host wrappers
void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y,
                 const c10::optional<at::Tensor>& rstd, double eps) {
  check_bf16_2d(x, "x");
  check_bf16_2d(w, "w");
  check_bf16_2d(y, "y");
  const int H = x.size(-1);
  const long rows = x.numel() / H;
  TORCH_CHECK(H % 8 == 0 && H <= kNormThreads * kMaxVecPerThread * 8, "rmsnorm: unsupported H");
  if (rows == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  const int nvec = H / 8;
  auto st = at::cuda::getCurrentCUDAStream();
  const int sms = num_sms(x.get_device());
#define KORE_RMS_FWD(T, V)                                                                           \
  rmsnorm_fwd_kernel<T, V><<<(int)std::min<long>(rows, (long)sms * (2048 / T)), T, 0, st>>>(          \
      (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(), \
      rstd ? rstd->data_ptr<float>() : nullptr, rows, H, (float)eps)
  if (nvec <= 256) KORE_RMS_FWD(256, 1);
  else if (nvec <= 512) KORE_RMS_FWD(256, 2);
  else if (nvec <= 768) KORE_RMS_FWD(256, 3);
  else if (nvec <= 1024) KORE_RMS_FWD(256, 4);
  else KORE_RMS_FWD(128, 8);
#undef KORE_RMS_FWD
  check_cuda(cudaGetLastError(), "rmsnorm_fwd");
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                 const at::Tensor& rstd, const c10::optional<at::Tensor>& dres, at::Tensor& dx,
                 const c10::optional<at::Tensor>& dw) {
  check_bf16_2d(dy, "dy");
  check_bf16_2d(x, "x");
  check_bf16_2d(dx, "dx");
  const int H = x.size(-1);
  const long rows = x.numel() / H;
  if (rows == 0) return;
  TORCH_CHECK(H % 8 == 0 && H <= 256 * 4 * 8, "rmsnorm_bwd: unsupported H");
  if (dw) TORCH_CHECK(dw->scalar_type() == at::kFloat && dw->numel() == H, "dw must be fp32 [H]");
  c10::cuda::CUDAGuard g(x.device());
  const int nvec = H / 8;
  auto st = at::cuda::getCurrentCUDAStream();
  const int sms = num_sms(x.get_device());
  // persistent blocks (two 256-thread blocks per SM) accumulate dw over their rows
#define KORE_RMS_BWD(T, V)                                                                           \
  rmsnorm_bwd_kernel<T, V><<<(int)std::min<long>(rows, (long)sms * (512 / T)), T, 0, st>>>(           \
      (const __nv_bfloat16*)dy.data_ptr(), (const __nv_bfloat16*)x.data_ptr(),                         \
      (const __nv_bfloat16*)w.data_ptr(), rstd.data_ptr<float>(),                                     \
      dres ? (const __nv_bfloat16*)dres->data_ptr() : nullptr, (__nv_bfloat16*)dx.data_ptr(),         \
      dw ? dw->data_ptr<float>() : nullptr, rows, H)
  if (nvec <= 256) KORE_RMS_BWD(256, 1);
  else if (nvec <= 512) KORE_RMS_BWD(256, 2);
  else if (nvec <= 768) KORE_RMS_BWD(256, 3);
  else KORE_RMS_BWD(256, 4);
#undef KORE_RMS_BWD
  check_cuda(cudaGetLastError(), "rmsnorm_bwd");
}

void qk_norm_rope_fwd(const at::Tensor& qkv, const at::Tensor& qw, const at::Tensor& kw,
                      const at::Tensor& pos, const at::Tensor& cos_t, const at::Tensor& sin_t,
                      at::Tensor& out, const c10::optional<at::Tensor>& rstd, int64_t Hq,
                      int64_t Hkv, double eps) {
  check_bf16_2d(qkv, "qkv");
  const long T = qkv.size(0);
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * Hkv) * 128, "qk_norm_rope: head_dim must be 128");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.numel() == T, "pos must be int32 [T]");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(qkv.device());
  TORCH_CHECK(Hq + Hkv <= 8 * kQkMaxHeadsPerWarp, "qk_norm_rope: at most 96 q + k heads");
  TORCH_CHECK(cos_t.stride(0) == 64 && sin_t.stride(0) == 64 && cos_t.stride(1) == 1 && sin_t.stride(1) == 1 &&
                  (reinterpret_cast<uintptr_t>(cos_t.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sin_t.data_ptr()) & 15) == 0,
              "qk_norm_rope: contiguous, 16-byte aligned [max_pos, 64] fp32 cos/sin tables");
  qk_norm_rope_fwd_kernel<<<(int)T, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)qkv.data_ptr(), (const __nv_bfloat16*)qw.data_ptr(),
      (const __nv_bfloat16*)kw.data_ptr(), pos.data_ptr<int>(), cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), (__nv_bfloat16*)out.data_ptr(),
      rstd ? rstd->data_ptr<float>() : nullptr, T, Hq, Hkv, (float)eps);
  check_cuda(cudaGetLastError(), "qk_norm_rope_fwd");
}

void qk_norm_rope_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& qw,
                      const at::Tensor& kw, const at::Tensor& pos, const at::Tensor& cos_t,
                      const at::Tensor& sin_t, at::Tensor& dqkv, at::Tensor& dqw, at::Tensor& dkw,
                      int64_t Hq, int64_t Hkv, double eps) {
  const long T = qkv.size(0);
  if (T == 0) return;
  TORCH_CHECK(dqw.scalar_type() == at::kFloat && dkw.scalar_type() == at::kFloat,
              "dqw/dkw must be fp32");
  c10::cuda::CUDAGuard g(qkv.device());
  const int threads = 256;
  const int grid = grid_for(T * (Hq + Hkv) * 32, threads, qkv.get_device());
  qk_norm_rope_bwd_kernel<<<grid, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)qkv.data_ptr(),
      (const __nv_bfloat16*)qw.data_ptr(), (const __nv_bfloat16*)kw.data_ptr(),
      pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
      (__nv_bfloat16*)dqkv.data_ptr(), dqw.data_ptr<float>(), dkw.data_ptr<float>(), T, Hq, Hkv,
      (float)eps);
  check_cuda(cudaGetLastError(), "qk_norm_rope_bwd");
}

void swiglu_fwd(const at::Tensor& gu, at::Tensor& out) {
  const long T = gu.size(0);
  const int F = gu.size(1) / 2;
  TORCH_CHECK(F % 8 == 0, "swiglu: F must be a multiple of 8");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(gu.device());
  swiglu_fwd_kernel<<<grid_for(T * F / 8, 256, gu.get_device()), 256, 0,
                      at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)out.data_ptr(), T, F, gu.stride(0));
  check_cuda(cudaGetLastError(), "swiglu_fwd");
}

void swiglu_bwd(const at::Tensor& dout, const at::Tensor& gu, at::Tensor& dgu) {
  const long T = gu.size(0);
  const int F = gu.size(1) / 2;
  if (T == 0) return;
  TORCH_CHECK(gu.stride(0) == dgu.stride(0), "swiglu_bwd: gu/dgu stride mismatch");
  c10::cuda::CUDAGuard g(gu.device());
  swiglu_bwd_kernel<<<grid_for(T * F / 8, 256, gu.get_device()), 256, 0,
                      at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)dout.data_ptr(), (const __nv_bfloat16*)gu.data_ptr(),
      (__nv_bfloat16*)dgu.data_ptr(), T, F, gu.stride(0));
  check_cuda(cudaGetLastError(), "swiglu_bwd");
}

void embed_fwd(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kLong, "ids must be int64");
  const long T = ids.numel();
  const int H = table.size(1);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(table.device());
  embed_fwd_kernel<<<grid_for(T * H / 8, 256, table.get_device()), 256, 0,
                     at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<long>(), (const __nv_bfloat16*)table.data_ptr(), (__nv_bfloat16*)out.data_ptr(),
      T, H);
  check_cuda(cudaGetLastError(), "embed_fwd");
}

void embed_bwd(const at::Tensor& ids, const at::Tensor& dy, at::Tensor& dtable) {
  const long T = ids.numel();
  const int H = dy.size(1);
  if (T == 0) return;
  c10::cuda::CUDAGuard g(dy.device());
  const int grid = grid_for(T * H / 8, 256, dy.get_device());
  auto st = at::cuda::getCurrentCUDAStream();
  if (dtable.scalar_type() == at::kFloat)
    embed_bwd_kernel<float><<<grid, 256, 0, st>>>(ids.data_ptr<long>(),
                                                  (const __nv_bfloat16*)dy.data_ptr(),
                                                  dtable.data_ptr<float>(), T, H);
  else if (dtable.scalar_type() == at::kBFloat16)
    embed_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        ids.data_ptr<long>(), (const __nv_bfloat16*)dy.data_ptr(),
        (__nv_bfloat16*)dtable.data_ptr(), T, H);
  else
    TORCH_CHECK(false, "embed_bwd: dtable must be fp32 or bf16");
  check_cuda(cudaGetLastError(), "embed_bwd");
}

}  // namespace kore
