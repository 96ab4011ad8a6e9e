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

// ---------------------------------------------------------------- device routing plan
// Expert-major layout with every expert's rows padded to a multiple of 64 (pad
// rows are zero inputs, so they produce zero outputs and zero weight-gradient
// terms): the grouped GEMMs' tiles and the weight gradient's 64-row K blocks
// never straddle two experts, and nothing of the plan returns to the host.
constexpr int kPlanThreads = 1024;
constexpr int kPad = 64;

KORE_DEV int block_excl_scan(int v, int* buf, int& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x / 32;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffff, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) buf[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = lane < (int)(blockDim.x / 32) ? buf[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffff, w, o);
      if (lane >= o) w += y;
    }
    buf[lane] = w;     // inclusive prefix of the warp totals
  }
  __syncthreads();
  total = buf[blockDim.x / 32 - 1];
  const int before = wid > 0 ? buf[wid - 1] : 0;
  __syncthreads();
  return before + x - v;
}

// counts[e - lo] = number of (token, slot) pairs routed to expert e, lo <= e < hi
__global__ void __launch_bounds__(kPlanThreads) plan_count_kernel(const int* __restrict__ idx, long P, int lo,
                                                                  int* __restrict__ counts) {
  const int e = lo + blockIdx.x;
  int c = 0;
  for (long i = threadIdx.x; i < P; i += blockDim.x) c += idx[i] == e;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffff, c, o);
  __shared__ int red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x / 32); ++w) t += red[w];
    counts[blockIdx.x] = t;
  }
}

// One block per local expert: its padded offset, the stable rank of each of
// its pairs (token order), pos[pair], the source token of every row of its
// padded block (-1 for pad rows), its 128-row tiles, and (last block) the
// totals. offsets has E_local + 1 entries.
__global__ void __launch_bounds__(kPlanThreads) plan_assign_kernel(
    const int* __restrict__ idx, long P, int k, int lo, int El, const int* __restrict__ counts,
    int* __restrict__ pos, int* __restrict__ src_row, int* __restrict__ offsets, int4* __restrict__ tiles,
    int* __restrict__ ntiles) {
  __shared__ int buf[32];
  __shared__ int s_off, s_tile0;
  const int el = blockIdx.x, e = lo + el;
  if (threadIdx.x == 0) {
    int off = 0, t0 = 0;
    for (int j = 0; j < el; ++j) {
      const int pc = (counts[j] + kPad - 1) / kPad * kPad;
      off += pc;
      t0 += (pc + 127) / 128;
    }
    s_off = off;
    s_tile0 = t0;
  }
  __syncthreads();
  const int off = s_off;
  const int cnt = counts[el];
  const int pcnt = (cnt + kPad - 1) / kPad * kPad;
  int base = 0;
  for (long c0 = 0; c0 < P; c0 += blockDim.x) {
    const long i = c0 + threadIdx.x;
    const int hit = (i < P && idx[i] == e) ? 1 : 0;
    int total;
    const int r = block_excl_scan(hit, buf, total) + base;
    if (hit) {
      pos[i] = off + r;
      src_row[off + r] = (int)(i / k);
    }
    base += total;
  }
  for (int r = cnt + threadIdx.x; r < pcnt; r += blockDim.x) src_row[off + r] = -1;
  const int nt = (pcnt + 127) / 128;
  for (int t = threadIdx.x; t < nt; t += blockDim.x)
    tiles[s_tile0 + t] = make_int4(el, off + 128 * t, off + pcnt, 0);
  if (threadIdx.x == 0) {
    offsets[el] = off;
    if (el == El - 1) {
      offsets[El] = off + pcnt;
      ntiles[0] = s_tile0 + nt;
    }
  }
}

// rows[r] = x[src_row[r]] (zero row for src_row < 0); H % 8 == 0
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ src_row,
                                   __nv_bfloat16* __restrict__ out, long R, int H) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;   // one thread per 8 elements
  const long per = H / 8;
  if (i >= R * per) return;
  const long r = i / per;
  const int c = (int)(i % per) * 8;
  const int s = src_row[r];
  uint4 v = make_uint4(0, 0, 0, 0);
  if (s >= 0) v = *reinterpret_cast<const uint4*>(x + (long)s * H + c);
  *reinterpret_cast<uint4*>(out + r * H + c) = v;
}

// Expert-parallel plan from the all-gathered per-rank counts (allc [W, E],
// int32, still on the device): for every pair of this rank its owner rank and
// row in the owner's receive buffer (owner blocks are laid out expert-major,
// each expert padded to 64 rows, source ranks in rank order inside an expert);
// for this rank's own experts the padded offsets, totals and grouped-GEMM
// tiles. A receive buffer smaller than an owner's rows sets *overflow.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(
    const int* __restrict__ idx, long P, const int* __restrict__ allc, int W, int E, int El, int rank, long cap,
    int* __restrict__ dst_rank, long* __restrict__ dst_row, int* __restrict__ loc_offsets,
    int* __restrict__ loc_totals, int4* __restrict__ tiles, int* __restrict__ ntiles, int* __restrict__ overflow) {
  __shared__ int buf[32];
  __shared__ long s_myoff, s_base, s_end;
  __shared__ int s_tile0;
  const int e = blockIdx.x, d = e / El;
  if (threadIdx.x == 0) {
    long base = 0, end = 0;
    int t0 = 0;
    for (int f = d * El; f < (d + 1) * El; ++f) {
      long tot = 0;
      for (int s = 0; s < W; ++s) tot += allc[s * E + f];
      const long pt = (tot + kPad - 1) / kPad * kPad;
      if (f < e) {
        base += pt;
        t0 += (int)((pt + 127) / 128);
      }
      end += pt;
    }
    long mine = base;
    for (int s = 0; s < rank; ++s) mine += allc[s * E + e];
    s_myoff = mine;
    s_base = base;
    s_end = end;
    s_tile0 = t0;
    if (e == (d + 1) * El - 1 && end > cap) atomicExch(overflow, 1);
  }
  __syncthreads();
  long rbase = 0;
  for (long c0 = 0; c0 < P; c0 += blockDim.x) {
    const long i = c0 + threadIdx.x;
    const int hit = (i < P && idx[i] == e) ? 1 : 0;
    int total;
    const int r = block_excl_scan(hit, buf, total);
    if (hit) {
      dst_rank[i] = d;
      dst_row[i] = s_myoff + rbase + r;
    }
    rbase += total;
  }
  if (d == rank && threadIdx.x == 0) {
    const int el = e - d * El;
    long tot = 0;
    for (int s = 0; s < W; ++s) tot += allc[s * E + e];
    const long pt = (tot + kPad - 1) / kPad * kPad;
    loc_offsets[el] = (int)s_base;
    loc_totals[el] = (int)tot;
    const int nt = (int)((pt + 127) / 128);
    for (int t = 0; t < nt; ++t) tiles[s_tile0 + t] = make_int4(el, (int)(s_base + 128 * t), (int)(s_base + pt), 0);
    if (el == El - 1) {
      loc_offsets[El] = (int)s_end;
      ntiles[0] = s_tile0 + nt;
    }
  }
}

// zero the pad rows [off + total, next offset) of every local expert's block
__global__ void zero_pad_rows_kernel(__nv_bfloat16* __restrict__ buf, const int* __restrict__ offsets,
                                     const int* __restrict__ totals, int H) {
  const int el = blockIdx.x;
  const long a = (long)offsets[el] + totals[el], b = offsets[el + 1];
  for (long i = (long)threadIdx.x * 8; i < (b - a) * H; i += (long)blockDim.x * 8)
    *reinterpret_cast<uint4*>(buf + a * H + i) = make_uint4(0, 0, 0, 0);
}

// pad entries [off + total, next offset) of every local expert's block of the
// pull-dispatch index: -1 (the staging copy zero-fills those rows)
__global__ void index_pads_kernel(int* __restrict__ index, const int* __restrict__ offsets,
                                  const int* __restrict__ totals, long cap) {
  const int el = blockIdx.x;
  const long a = (long)offsets[el] + totals[el], b = min((long)offsets[el + 1], cap);
  for (long i = a + threadIdx.x; i < b; i += blockDim.x) index[i] = -1;
}

inline int warps_grid(long n, int warps_per_block = 8) {
  return (int)((n + warps_per_block - 1) / warps_per_block);
}

}  // namespace moe

// Device routing plan (no host synchronisation): idx int32 [T, k] expert ids;
// local experts [lo, hi). Outputs: pos int32 [T * k] (padded expert-major row of
// each pair, -1 for experts outside the range), src_row int32 [cap_rows],
// offsets int32 [hi - lo + 1], tiles int32 [cap_tiles * 4], ntiles int32 [1],
// counts int32 [hi - lo]. cap_rows >= T * k + (hi - lo) * 63.
void moe_plan(const at::Tensor& idx, int64_t lo, int64_t hi, at::Tensor& pos, at::Tensor& src_row,
              at::Tensor& offsets, at::Tensor& tiles, at::Tensor& ntiles, at::Tensor& counts) {
  TORCH_CHECK(idx.scalar_type() == at::kInt && idx.is_contiguous() && idx.dim() == 2, "idx int32 [T, k]");
  const long P = idx.numel();
  const int k = idx.size(1);
  const int El = (int)(hi - lo);
  TORCH_CHECK(El > 0 && counts.numel() >= El && offsets.numel() >= El + 1 && pos.numel() >= P, "plan sizes");
  TORCH_CHECK(src_row.numel() >= P + (long)El * (moe::kPad - 1), "src_row capacity");
  TORCH_CHECK(tiles.numel() / 4 >= (P + (long)El * (moe::kPad - 1)) / 128 + El, "tile capacity");
  c10::cuda::CUDAGuard g(idx.device());
  auto st = at::cuda::getCurrentCUDAStream();
  pos.fill_(-1);
  src_row.fill_(-1);   // rows past the last expert's padded block stay pad rows
  moe::plan_count_kernel<<<El, moe::kPlanThreads, 0, st>>>(idx.data_ptr<int>(), P, (int)lo, counts.data_ptr<int>());
  check_cuda(cudaGetLastError(), "moe plan count");
  moe::plan_assign_kernel<<<El, moe::kPlanThreads, 0, st>>>(
      idx.data_ptr<int>(), P, k, (int)lo, El, counts.data_ptr<int>(), pos.data_ptr<int>(),
      src_row.data_ptr<int>(), offsets.data_ptr<int>(), reinterpret_cast<int4*>(tiles.data_ptr<int>()),
      ntiles.data_ptr<int>());
  check_cuda(cudaGetLastError(), "moe plan assign");
}

void moe_ep_plan(const at::Tensor& idx, const at::Tensor& allc, int64_t W, int64_t rank, int64_t cap,
                 at::Tensor& dst_rank, at::Tensor& dst_row, at::Tensor& loc_offsets, at::Tensor& loc_totals,
                 at::Tensor& tiles, at::Tensor& ntiles, at::Tensor& overflow) {
  TORCH_CHECK(idx.scalar_type() == at::kInt && allc.scalar_type() == at::kInt && dst_row.scalar_type() == at::kLong,
              "ep plan dtypes");
  const long P = idx.numel();
  const int E = (int)(allc.numel() / W), El = E / (int)W;
  TORCH_CHECK(E % W == 0 && loc_offsets.numel() >= El + 1 && loc_totals.numel() >= El, "ep plan sizes");
  c10::cuda::CUDAGuard g(idx.device());
  moe::ep_plan_kernel<<<E, moe::kPlanThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int>(), P, allc.data_ptr<int>(), (int)W, E, El, (int)rank, cap, dst_rank.data_ptr<int>(),
      dst_row.data_ptr<long>(), loc_offsets.data_ptr<int>(), loc_totals.data_ptr<int>(),
      reinterpret_cast<int4*>(tiles.data_ptr<int>()), ntiles.data_ptr<int>(), overflow.data_ptr<int>());
  check_cuda(cudaGetLastError(), "moe ep plan");
}

void moe_zero_pad_rows(at::Tensor& buf, const at::Tensor& offsets, const at::Tensor& totals, int64_t H) {
  const int El = totals.numel();
  if (El == 0) return;
  c10::cuda::CUDAGuard g(buf.device());
  moe::zero_pad_rows_kernel<<<El, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (__nv_bfloat16*)buf.data_ptr(), offsets.data_ptr<int>(), totals.data_ptr<int>(), (int)H);
  check_cuda(cudaGetLastError(), "moe zero pad rows");
}

void moe_index_pads(at::Tensor& index, const at::Tensor& offsets, const at::Tensor& totals) {
  TORCH_CHECK(index.scalar_type() == at::kInt && offsets.scalar_type() == at::kInt &&
                  totals.scalar_type() == at::kInt && index.is_cuda(), "index pads: int32 device tensors");
  const int El = totals.numel();
  if (El == 0) return;
  c10::cuda::CUDAGuard g(index.device());
  moe::index_pads_kernel<<<El, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      index.data_ptr<int>(), offsets.data_ptr<int>(), totals.data_ptr<int>(), (long)index.numel());
  check_cuda(cudaGetLastError(), "moe index pads");
}

void moe_gather_rows(const at::Tensor& x, const at::Tensor& src_row, at::Tensor& out) {
  const long R = src_row.numel();
  const int H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && x.is_contiguous() && out.is_contiguous() && out.size(0) >= R, "gather rows layout");
  if (R == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  const long n = R * H / 8;
  moe::gather_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), src_row.data_ptr<int>(), (__nv_bfloat16*)out.data_ptr(), R, H);
  check_cuda(cudaGetLastError(), "moe gather rows");
}

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
