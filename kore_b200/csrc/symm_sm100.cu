// Symmetric peer memory over NVLink/NVSwitch and the fused collective kernels
// of the sharded optimizer.
//
// SymmetricHeap: one cudaMalloc'd region per rank, exported with a CUDA IPC
// handle, exchanged over the process group by the Python side, and mapped on
// every peer (cudaIpcOpenMemHandle). Tensors carved from the heap therefore
// have the same offset on every rank, and kernels address a peer's copy as
// peer_base[p] + offset with plain loads/stores over NVLink.
//
// Kernels (all waits bounded; a timeout records error code 2 and returns):
//   * symm_barrier:    epoch-tagged flag barrier across ranks
//                      (st.release.sys / ld.acquire.sys)
//   * rs_sumsq:        reduce-scatter of bf16 gradients (this rank's shard, summed
//                      over all peers' full gradient buffers with P2P loads) into
//                      an fp32 shard, fused with the sum of squares for clipping
//   * scalar_allreduce: every rank publishes its partial sum-of-squares to all
//                      peers; each rank then sums the world's values
//   * adamw_bcast:     AdamW on the fp32 shard (global-norm clip read on device),
//                      then the new bf16 parameters are stored straight into every
//                      peer's parameter buffer (the all-gather fused into the
//                      update, path b of the north star).
// No TMA and no multicast loads touch peer memory here.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstring>
#include <memory>
#include <vector>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace symm {

constexpr int kMaxWorld = 8;

struct PeerPtrs {
  char* p[kMaxWorld];
};

KORE_DEV void st_release_sys(unsigned long long* a, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
KORE_DEV unsigned long long ld_acquire_sys(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// Wait until *a >= want (epoch compare on the high 32 bits). Bounded.
KORE_DEV bool wait_epoch(const unsigned long long* a, unsigned int want) {
  uint64_t t0 = 0;
  for (int it = 0;; ++it) {
    unsigned long long v = ld_acquire_sys(a);
    if ((unsigned int)(v >> 32) >= want) return true;
    if (it == 64) t0 = globaltimer();
    if (it > 64 && globaltimer() - t0 > kWaitTimeoutNs) {
      atomicExch(&g_error, 2);
      return false;
    }
  }
}

// signal pad layout (per rank, in the heap): slot[0..world) barrier flags,
// slot[16..16+world) scalar all-reduce values.
__global__ void barrier_kernel(PeerPtrs sig, int rank, int world, unsigned int epoch,
                               unsigned long long sig_off) {
  const int p = threadIdx.x;
  if (p < world) {
    __threadfence_system();
    unsigned long long* remote = reinterpret_cast<unsigned long long*>(sig.p[p] + sig_off) + rank;
    st_release_sys(remote, ((unsigned long long)epoch) << 32);
    const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(sig.p[rank] + sig_off) + p;
    wait_epoch(mine, epoch);
  }
}

template <int W>
__global__ void rs_sumsq_kernel(PeerPtrs grads, long shard_off, long n, float* __restrict__ out,
                                float* __restrict__ sumsq, float scale) {
  float acc = 0.f;
  const long nvec = n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < W; ++p) {
      const uint4 u = *reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(grads.p[p]) + shard_off + i * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        s[2 * e] += f.x;
        s[2 * e + 1] += f.y;
      }
    }
    if (out != nullptr) {
      *reinterpret_cast<float4*>(out + i * 8) =
          make_float4(s[0] * scale, s[1] * scale, s[2] * scale, s[3] * scale);
      *reinterpret_cast<float4*>(out + i * 8 + 4) =
          make_float4(s[4] * scale, s[5] * scale, s[6] * scale, s[7] * scale);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += s[e] * scale * s[e] * scale;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) t += red[i];
    atomicAdd(sumsq, t);
  }
}

// Publish local value to every peer's slot[16 + rank]; wait for all and sum.
__global__ void scalar_allreduce_kernel(PeerPtrs sig, int rank, int world, unsigned int epoch,
                                        unsigned long long sig_off, const float* __restrict__ local,
                                        float* __restrict__ out) {
  __shared__ float vals[kMaxWorld];
  const int p = threadIdx.x;
  if (p < world) {
    const float v = *local;
    unsigned long long* remote = reinterpret_cast<unsigned long long*>(sig.p[p] + sig_off) + 16 + rank;
    st_release_sys(remote, (((unsigned long long)epoch) << 32) | __float_as_uint(v));
    const unsigned long long* mine = reinterpret_cast<const unsigned long long*>(sig.p[rank] + sig_off) + 16 + p;
    float got = 0.f;
    if (wait_epoch(mine, epoch)) got = __uint_as_float((unsigned int)(ld_acquire_sys(mine) & 0xffffffffu));
    vals[p] = got;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < world; ++i) t += vals[i];
    *out = t;
  }
}

KORE_DEV uint32_t hash32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

template <int W>
__global__ void adamw_bcast_kernel(PeerPtrs grads, float gscale, float* __restrict__ master,
                                   float* __restrict__ m, float* __restrict__ v, PeerPtrs params,
                                   long shard_off, long n, float lr, float b1, float b2, float eps,
                                   float wd, float bc1, float bc2, const float* __restrict__ sumsq,
                                   float max_norm, uint32_t seed) {
  float scale = 1.f;
  if (sumsq != nullptr && max_norm > 0.f) scale = fminf(1.f, max_norm / (sqrtf(*sumsq) + 1e-6f));
  const long nvec = n / 8;
  const __nv_bfloat16* own = reinterpret_cast<const __nv_bfloat16*>(params.p[0]);  // slot 0 = this rank
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    uint32_t packed[4];
    float gs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < W; ++p) {  // reduce-scatter fused into the update: P2P loads
      const uint4 u = *reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(grads.p[p]) + shard_off + i * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        gs[2 * e] += f.x;
        gs[2 * e + 1] += f.y;
      }
    }
    const uint4 cur = *reinterpret_cast<const uint4*>(own + shard_off + i * 8);
    const __nv_bfloat162* ch = reinterpret_cast<const __nv_bfloat162*>(&cur);
    // fp32 state as two 16-byte vectors per thread (8 consecutive elements)
    float4* m4 = reinterpret_cast<float4*>(m + i * 8);
    float4* v4 = reinterpret_cast<float4*>(v + i * 8);
    float4* w4 = master ? reinterpret_cast<float4*>(master + i * 8) : nullptr;
    float mv[8], vv[8], wv[8];
    {
      const float4 a = m4[0], b = m4[1], c = v4[0], d = v4[1];
      mv[0] = a.x; mv[1] = a.y; mv[2] = a.z; mv[3] = a.w; mv[4] = b.x; mv[5] = b.y; mv[6] = b.z; mv[7] = b.w;
      vv[0] = c.x; vv[1] = c.y; vv[2] = c.z; vv[3] = c.w; vv[4] = d.x; vv[5] = d.y; vv[6] = d.z; vv[7] = d.w;
      if (w4) {
        const float4 e = w4[0], f = w4[1];
        wv[0] = e.x; wv[1] = e.y; wv[2] = e.z; wv[3] = e.w; wv[4] = f.x; wv[5] = f.y; wv[6] = f.z; wv[7] = f.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 cf = __bfloat1622float2(ch[e]);
          wv[2 * e] = cf.x;
          wv[2 * e + 1] = cf.y;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float gi = gs[k] * gscale * scale;
      mv[k] = b1 * mv[k] + (1.f - b1) * gi;
      vv[k] = b2 * vv[k] + (1.f - b2) * gi * gi;
      wv[k] = wv[k] * (1.f - lr * wd) - lr * (mv[k] / bc1) / (sqrtf(vv[k] / bc2) + eps);
    }
    m4[0] = make_float4(mv[0], mv[1], mv[2], mv[3]);
    m4[1] = make_float4(mv[4], mv[5], mv[6], mv[7]);
    v4[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
    v4[1] = make_float4(vv[4], vv[5], vv[6], vv[7]);
    if (w4) {
      w4[0] = make_float4(wv[0], wv[1], wv[2], wv[3]);
      w4[1] = make_float4(wv[4], wv[5], wv[6], wv[7]);
    }
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      float w2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const long j = i * 8 + e + k;
        if (w4) {
          w2[k] = wv[e + k];
        } else {  // stochastic rounding to bf16 (unbiased)
          uint32_t b = __float_as_uint(wv[e + k]);
          b += hash32((uint32_t)(shard_off + j) * 0x9E3779B9u ^ seed) & 0xffffu;
          w2[k] = __uint_as_float(b & 0xffff0000u);
        }
      }
      packed[e / 2] = pack_bf16(w2[0], w2[1]);
    }
    const uint4 out = make_uint4(packed[0], packed[1], packed[2], packed[3]);
#pragma unroll
    for (int p = 0; p < W; ++p)
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(params.p[p]) + shard_off + i * 8) = out;
  }
}

// ------------------------------------------------------------------ heap
struct Heap {
  int device = -1;
  int rank = 0, world = 1;
  char* base = nullptr;
  size_t bytes = 0;
  std::vector<char*> peers;  // peers[p] = base of rank p's heap mapped here (peers[rank] = base)
};

}  // namespace symm

// Python-facing handle (opaque int id).
static std::vector<std::unique_ptr<symm::Heap>> g_heaps;

int64_t symm_heap_create(int64_t bytes, int64_t rank, int64_t world) {
  TORCH_CHECK(world >= 1 && world <= symm::kMaxWorld, "world must be 1..8");
  auto h = std::make_unique<symm::Heap>();
  check_cuda(cudaGetDevice(&h->device), "cudaGetDevice");
  h->rank = rank;
  h->world = world;
  h->bytes = (size_t)bytes;
  void* p = nullptr;
  check_cuda(cudaMalloc(&p, h->bytes), "symm heap cudaMalloc");
  check_cuda(cudaMemset(p, 0, h->bytes), "symm heap memset");
  h->base = static_cast<char*>(p);
  h->peers.assign(world, nullptr);
  h->peers[rank] = h->base;
  g_heaps.push_back(std::move(h));
  return (int64_t)g_heaps.size() - 1;
}

// The 64-byte cudaIpcMemHandle_t as a uint8 CPU tensor.
at::Tensor symm_heap_handle(int64_t id) {
  auto& h = g_heaps.at(id);
  cudaIpcMemHandle_t hd;
  check_cuda(cudaIpcGetMemHandle(&hd, h->base), "cudaIpcGetMemHandle");
  auto t = at::empty({(int64_t)sizeof(hd)}, at::kByte);
  std::memcpy(t.data_ptr(), &hd, sizeof(hd));
  return t;
}

// handles: uint8 [world, 64] from all ranks (row r = rank r).
void symm_heap_open(int64_t id, const at::Tensor& handles) {
  auto& h = g_heaps.at(id);
  TORCH_CHECK(handles.size(0) == h->world && handles.size(1) == (int64_t)sizeof(cudaIpcMemHandle_t),
              "handles must be [world, 64]");
  auto hc = handles.contiguous();
  for (int p = 0; p < h->world; ++p) {
    if (p == h->rank) continue;
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, hc.data_ptr<uint8_t>() + p * sizeof(hd), sizeof(hd));
    void* ptr = nullptr;
    check_cuda(cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    h->peers[p] = static_cast<char*>(ptr);
  }
}

// A tensor view of the local heap at a byte offset (no ownership).
at::Tensor symm_heap_tensor(int64_t id, int64_t offset, const std::vector<int64_t>& shape,
                            at::ScalarType dtype) {
  auto& h = g_heaps.at(id);
  int64_t n = 1;
  for (auto s : shape) n *= s;
  TORCH_CHECK(offset >= 0 && offset % 256 == 0 &&
                  (size_t)(offset + n * (int64_t)c10::elementSize(dtype)) <= h->bytes,
              "symm tensor out of heap bounds");
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, h->device);
  return at::from_blob(h->base + offset, shape, [](void*) {}, opts);
}

static symm::PeerPtrs peer_ptrs(const symm::Heap& h, int64_t offset, bool self_first) {
  symm::PeerPtrs pp;
  for (int i = 0; i < symm::kMaxWorld; ++i) pp.p[i] = nullptr;
  for (int p = 0; p < h.world; ++p) {
    const int idx = self_first ? (p == 0 ? h.rank : (p <= h.rank ? p - 1 : p)) : p;
    pp.p[p] = h.peers[idx] + offset;
  }
  return pp;
}

void symm_barrier(int64_t id, int64_t sig_offset, int64_t epoch) {
  auto& h = *g_heaps.at(id);
  symm::PeerPtrs sig = peer_ptrs(h, 0, false);
  symm::barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(sig, h.rank, h.world, (unsigned)epoch,
                                                                        (unsigned long long)sig_offset);
  check_cuda(cudaGetLastError(), "symm_barrier");
}

// grads: heap offset of the FULL bf16 gradient buffer (same on every rank);
// this rank's shard [rank*n, (rank+1)*n) is summed over peers into out (fp32).
void symm_rs_sumsq(int64_t id, int64_t grad_offset, int64_t n, const c10::optional<at::Tensor>& out,
                   at::Tensor& sumsq, double scale) {
  auto& h = *g_heaps.at(id);
  TORCH_CHECK(n % 8 == 0, "shard length must be a multiple of 8");
  symm::PeerPtrs g = peer_ptrs(h, grad_offset, false);
  const long shard_off = (long)h.rank * n;
  const int grid = (int)std::min<long>((n / 8 + 255) / 256, (long)num_sms(h.device) * 4);
  auto st = at::cuda::getCurrentCUDAStream();
#define KORE_RS(W) symm::rs_sumsq_kernel<W><<<grid, 256, 0, st>>>(g, shard_off, n, out ? out->data_ptr<float>() : nullptr, \
                                                                  sumsq.data_ptr<float>(), (float)scale)
  switch (h.world) {
    case 1: KORE_RS(1); break;
    case 2: KORE_RS(2); break;
    case 4: KORE_RS(4); break;
    case 8: KORE_RS(8); break;
    default: TORCH_CHECK(false, "world must be 1, 2, 4 or 8");
  }
#undef KORE_RS
  check_cuda(cudaGetLastError(), "symm_rs_sumsq");
}

void symm_scalar_allreduce(int64_t id, int64_t sig_offset, int64_t epoch, const at::Tensor& local,
                           at::Tensor& out) {
  auto& h = *g_heaps.at(id);
  symm::PeerPtrs sig = peer_ptrs(h, 0, false);
  symm::scalar_allreduce_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      sig, h.rank, h.world, (unsigned)epoch, (unsigned long long)sig_offset, local.data_ptr<float>(),
      out.data_ptr<float>());
  check_cuda(cudaGetLastError(), "symm_scalar_allreduce");
}

void symm_adamw_bcast(int64_t id, int64_t param_offset, int64_t grad_offset, int64_t n, double gscale,
                      const c10::optional<at::Tensor>& master, at::Tensor& m, at::Tensor& v, double lr,
                      double b1, double b2, double eps, double wd, int64_t step,
                      const c10::optional<at::Tensor>& sumsq, double max_norm, int64_t seed) {
  auto& h = *g_heaps.at(id);
  TORCH_CHECK(n % 8 == 0, "shard length must be a multiple of 8");
  auto vec_ok = [&](const at::Tensor& t) {
    return t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous() && t.numel() >= n &&
           reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0;
  };
  TORCH_CHECK(vec_ok(m) && vec_ok(v) && (!master || vec_ok(*master)),
              "symm_adamw_bcast: m / v / master must be contiguous fp32, >= n elements, 16-byte aligned");
  TORCH_CHECK((param_offset % 16 == 0) && (grad_offset % 16 == 0), "symm_adamw_bcast: 16-byte aligned offsets");
  symm::PeerPtrs prm = peer_ptrs(h, param_offset, true);  // slot 0 = own buffer
  symm::PeerPtrs grd = peer_ptrs(h, grad_offset, false);
  const long shard_off = (long)h.rank * n;
  const float bc1 = 1.f - std::pow((float)b1, (float)step);
  const float bc2 = 1.f - std::pow((float)b2, (float)step);
  const int grid = (int)std::min<long>((n / 8 + 255) / 256, (long)num_sms(h.device) * 4);
  auto st = at::cuda::getCurrentCUDAStream();
  float* mp = master ? master->data_ptr<float>() : nullptr;
  const float* sq = sumsq ? sumsq->data_ptr<float>() : nullptr;
#define KORE_AB(W)                                                                                  \
  symm::adamw_bcast_kernel<W><<<grid, 256, 0, st>>>(grd, (float)gscale, mp, m.data_ptr<float>(),    \
                                                    v.data_ptr<float>(), prm, shard_off, n, lr, b1, b2, \
                                                    eps, wd, bc1, bc2, sq, max_norm, (uint32_t)seed)
  switch (h.world) {
    case 1: KORE_AB(1); break;
    case 2: KORE_AB(2); break;
    case 4: KORE_AB(4); break;
    case 8: KORE_AB(8); break;
    default: TORCH_CHECK(false, "world must be 1, 2, 4 or 8");
  }
#undef KORE_AB
  check_cuda(cudaGetLastError(), "symm_adamw_bcast");
}

}  // namespace kore

// ============================================================== expert-parallel rows
namespace kore {
namespace symm {

// Row scatter to peers: for pair i, row src_row[i] of the local matrix x [*, H]
// (times scale[i] when given) is stored into peer dst_rank[i]'s buffer at row
// dst_row[i] (P2P stores over NVLink). One warp per pair, 16-byte vectors.
__global__ void ep_scatter_kernel(const __nv_bfloat16* __restrict__ x, const long* __restrict__ src_row,
                                  const int* __restrict__ dst_rank, const long* __restrict__ dst_row,
                                  const float* __restrict__ scale, PeerPtrs dst, int n, int H, long cap) {
  const long i = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (i >= n) return;
  if (cap > 0 && dst_row[i] >= cap) return;     // receive buffer too small: the plan flagged it
  const __nv_bfloat16* s = x + src_row[i] * (long)H;
  __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dst.p[dst_rank[i]]) + dst_row[i] * (long)H;
  const float sc = scale ? scale[i] : 1.f;
  for (int c = lane * 8; c < H; c += 256) {
    uint4 u = *reinterpret_cast<const uint4*>(s + c);
    if (scale) {
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        h[e] = __floats2bfloat162_rn(f.x * sc, f.y * sc);
      }
    }
    *reinterpret_cast<uint4*>(d + c) = u;
  }
}

// Pull-dispatch index: pair i (token i / k) tells its owner which row of
// which rank's token buffer lands in receive row dst_row[i]:
// owner.index[dst_row[i]] = rank << 26 | (i / k). 4 bytes cross NVLink per pair.
__global__ void ep_index_push_kernel(PeerPtrs dst, const int* __restrict__ dst_rank,
                                     const long* __restrict__ dst_row, int n, int k, int rank, long cap) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const long r = dst_row[i];
  if (r >= cap) return;                      // receive buffer too small: the plan flagged it
  reinterpret_cast<int*>(dst.p[dst_rank[i]])[r] = (rank << 26) | (i / k);
}

// Pull-combine from peers: y[t] = sum_j w[t,j] * peer[rank[t,j]][row[t,j]] (+ resid[t]);
// with dw != nullptr also dw[t,j] = <g[t], peer row> (the combine backward's weight grad).
__global__ void ep_gather_kernel(PeerPtrs src, const int* __restrict__ rank, const long* __restrict__ row,
                                 const float* __restrict__ w, const __nv_bfloat16* __restrict__ resid,
                                 __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ g,
                                 float* __restrict__ dw, int T, int k, int H) {
  const long t = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  if (dw != nullptr) {
    for (int j = 0; j < k; ++j) {
      const __nv_bfloat16* pr = reinterpret_cast<const __nv_bfloat16*>(src.p[rank[t * k + j]]) + row[t * k + j] * (long)H;
      float dot = 0.f;
      for (int c = lane * 8; c < H; c += 256) {
        const uint4 a = *reinterpret_cast<const uint4*>(pr + c);
        const uint4 b = *reinterpret_cast<const uint4*>(g + t * H + c);
        const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float2 fa = __bfloat1622float2(ha[e]), fb = __bfloat1622float2(hb[e]);
          dot += fa.x * fb.x + fa.y * fb.y;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffff, dot, o);
      if (lane == 0) dw[t * k + j] = dot;
    }
    return;
  }
  for (int c = lane * 8; c < H; c += 256) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (resid) {
      const uint4 u = *reinterpret_cast<const uint4*>(resid + t * H + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] = f.x;
        acc[2 * e + 1] = f.y;
      }
    }
    for (int j = 0; j < k; ++j) {
      const float ww = w ? w[t * k + j] : 1.f;
      const __nv_bfloat16* pr = reinterpret_cast<const __nv_bfloat16*>(src.p[rank[t * k + j]]) + row[t * k + j] * (long)H;
      const uint4 u = *reinterpret_cast<const uint4*>(pr + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += ww * f.x;
        acc[2 * e + 1] += ww * f.y;
      }
    }
    *reinterpret_cast<uint4*>(y + t * H + c) =
        make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                   pack_bf16(acc[6], acc[7]));
  }
}

}  // namespace symm

void symm_ep_scatter(int64_t id, int64_t buf_offset, const at::Tensor& x, const at::Tensor& src_row,
                     const at::Tensor& dst_rank, const at::Tensor& dst_row,
                     const c10::optional<at::Tensor>& scale, int64_t cap) {
  auto& h = *g_heaps.at(id);
  const int n = src_row.numel(), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && x.is_contiguous(), "ep_scatter: contiguous rows, H % 8");
  if (n == 0) return;
  symm::PeerPtrs dst = peer_ptrs(h, buf_offset, false);
  symm::ep_scatter_kernel<<<(n + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)x.data_ptr(), src_row.data_ptr<long>(), dst_rank.data_ptr<int>(),
      dst_row.data_ptr<long>(), scale ? scale->data_ptr<float>() : nullptr, dst, n, H, (long)cap);
  check_cuda(cudaGetLastError(), "ep_scatter");
}

void symm_ep_index_push(int64_t id, int64_t index_offset, const at::Tensor& dst_rank, const at::Tensor& dst_row,
                        int64_t k, int64_t cap) {
  auto& h = *g_heaps.at(id);
  const int n = dst_rank.numel();
  TORCH_CHECK(dst_rank.scalar_type() == at::kInt && dst_row.scalar_type() == at::kLong && dst_row.numel() == n,
              "ep_index_push: dst_rank int32, dst_row int64 of equal length");
  TORCH_CHECK(index_offset % 4 == 0 && n / k < (1 << 26) && h.world <= 32, "ep_index_push: offsets and ranges");
  if (n == 0) return;
  symm::PeerPtrs dst = peer_ptrs(h, index_offset, false);
  symm::ep_index_push_kernel<<<(n + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      dst, dst_rank.data_ptr<int>(), dst_row.data_ptr<long>(), n, (int)k, h.rank, (long)cap);
  check_cuda(cudaGetLastError(), "ep_index_push");
}

void symm_ep_gather(int64_t id, int64_t buf_offset, const at::Tensor& rank, const at::Tensor& row,
                    const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& resid,
                    at::Tensor& y, const c10::optional<at::Tensor>& g, const c10::optional<at::Tensor>& dw,
                    int64_t H) {
  auto& h = *g_heaps.at(id);
  const int T = rank.size(0), k = rank.size(1);
  if (T == 0) return;
  symm::PeerPtrs src = peer_ptrs(h, buf_offset, false);
  symm::ep_gather_kernel<<<(T + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      src, rank.data_ptr<int>(), row.data_ptr<long>(), w ? w->data_ptr<float>() : nullptr,
      resid ? (const __nv_bfloat16*)resid->data_ptr() : nullptr, (__nv_bfloat16*)y.data_ptr(),
      g ? (const __nv_bfloat16*)g->data_ptr() : nullptr, dw ? dw->data_ptr<float>() : nullptr, T, k, (int)H);
  check_cuda(cudaGetLastError(), "ep_gather");
}

}  // namespace kore

// ============================================================== TP reduce + residual + RMSNorm
namespace kore {
namespace symm {

// x[r] += sum_w slots[w][r] (the reduce of GEMM->reduce-scatter), then
// hn[r] = rmsnorm(x[r]) * g. One CTA (128 threads) per local row; H <= 8192.
__global__ void tp_reduce_norm_kernel(const __nv_bfloat16* __restrict__ slots, int W, int R, int H,
                                      __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ g,
                                      __nv_bfloat16* __restrict__ hn, float eps) {
  const int r = blockIdx.x;
  __shared__ float red[4];
  float v[8][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = (threadIdx.x + i * 128) * 8;
    if (c < H) {
      float a[8];
      const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)r * H + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) { float2 f = __bfloat1622float2(h[e]); a[2 * e] = f.x; a[2 * e + 1] = f.y; }
      for (int w = 0; w < W; ++w) {
        const uint4 q = *reinterpret_cast<const uint4*>(slots + ((size_t)w * R + r) * H + c);
        const __nv_bfloat162* hq = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
        for (int e = 0; e < 4; ++e) { float2 f = __bfloat1622float2(hq[e]); a[2 * e] += f.x; a[2 * e + 1] += f.y; }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) { v[i][e] = a[e]; ss += a[e] * a[e]; }
      *reinterpret_cast<uint4*>(x + (size_t)r * H + c) =
          make_uint4(pack_bf16(a[0], a[1]), pack_bf16(a[2], a[3]), pack_bf16(a[4], a[5]), pack_bf16(a[6], a[7]));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffff, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  const float rs = rsqrtf((red[0] + red[1] + red[2] + red[3]) / H + eps);
  if (hn == nullptr) return;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = (threadIdx.x + i * 128) * 8;
    if (c < H) {
      const uint4 u = *reinterpret_cast<const uint4*>(g + c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
      float o[8];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 f = __bfloat1622float2(h[e]);
        o[2 * e] = v[i][2 * e] * rs * f.x;
        o[2 * e + 1] = v[i][2 * e + 1] * rs * f.y;
      }
      *reinterpret_cast<uint4*>(hn + (size_t)r * H + c) =
          make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
    }
  }
}

}  // namespace symm

void tp_reduce_norm(const at::Tensor& slots, int64_t W, int64_t R, at::Tensor& x, const c10::optional<at::Tensor>& g,
                    const c10::optional<at::Tensor>& hn, double eps) {
  const int H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8192 && x.is_contiguous(), "tp_reduce_norm: H % 8, H <= 8192");
  if (R == 0) return;
  symm::tp_reduce_norm_kernel<<<(int)R, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)slots.data_ptr(), (int)W, (int)R, H, (__nv_bfloat16*)x.data_ptr(),
      g ? (const __nv_bfloat16*)g->data_ptr() : nullptr, hn ? (__nv_bfloat16*)hn->data_ptr() : nullptr, (float)eps);
  check_cuda(cudaGetLastError(), "tp_reduce_norm");
}

// Device addresses of every peer's mapping of this heap at a byte offset.
std::vector<int64_t> symm_peer_addrs(int64_t id, int64_t offset) {
  auto& h = *g_heaps.at(id);
  std::vector<int64_t> out;
  for (int p = 0; p < h.world; ++p) out.push_back(reinterpret_cast<int64_t>(h.peers[p] + offset));
  return out;
}

// All-gather on the copy engines: for every rank p, ``bytes`` from peer p's
// heap at ``src_offset`` into ``dst`` at p * bytes, one cudaMemcpyAsync per
// rank on the current stream (NVLink peer copies, no SM time). The caller
// orders the copies after the peers wrote their shards (a device barrier or a
// collective) and before the peers overwrite them.
void symm_gather_ce(int64_t id, int64_t src_offset, int64_t bytes, at::Tensor& dst) {
  auto& h = *g_heaps.at(id);
  TORCH_CHECK(dst.is_cuda() && dst.is_contiguous(), "gather dst must be contiguous CUDA");
  TORCH_CHECK((int64_t)dst.numel() * dst.element_size() >= bytes * h.world, "gather dst too small");
  TORCH_CHECK(src_offset >= 0 && (size_t)(src_offset + bytes) <= h.bytes, "gather source outside the heap");
  c10::cuda::CUDAGuard g(dst.device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  uint8_t* out = reinterpret_cast<uint8_t*>(dst.data_ptr());
  for (int p = 0; p < h.world; ++p) {
    // start with this rank's own shard: the local copy finishes while the peers' stream in
    const int q = (h.rank + p) % h.world;
    check_cuda(cudaMemcpyAsync(out + (size_t)q * bytes, h.peers[q] + src_offset, bytes, cudaMemcpyDeviceToDevice, st),
               "symm gather copy");
  }
}

}  // namespace kore

// ============================================================== bounded flag wait (health check)
namespace kore {
namespace symm {

// Wait until *flag >= want or timeout_ns elapse; status 0 = seen, 2 = timed
// out. The same bounded-spin discipline as every peer wait in this file: the
// kernel always returns, the context stays usable and the host reads status.
__global__ void wait_flag_kernel(const unsigned long long* flag, unsigned long long want, unsigned long long timeout_ns,
                                 int* status) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (ld_acquire_sys(flag) >= want) { *status = 0; return; }
    if (globaltimer() - t0 > timeout_ns) { *status = 2; return; }
    __nanosleep(1000);
  }
}

}  // namespace symm

// Host: returns the wait status (0 seen, 2 timed out). ``flag`` is a uint64
// (int64 tensor) in device memory, local or a peer's mapping.
int64_t device_wait_flag(const at::Tensor& flag, int64_t want, double timeout_s) {
  TORCH_CHECK(flag.is_cuda() && flag.scalar_type() == at::kLong && flag.numel() >= 1, "device_wait_flag: int64 cuda");
  TORCH_CHECK(timeout_s > 0 && timeout_s <= 10.0, "device_wait_flag: timeout in (0, 10] s");
  auto st = at::full({1}, -1, flag.options().dtype(at::kInt));
  symm::wait_flag_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const unsigned long long*)flag.data_ptr(), (unsigned long long)want,
      (unsigned long long)(timeout_s * 1e9), st.data_ptr<int>());
  check_cuda(cudaGetLastError(), "device_wait_flag");
  return st.item<int>();
}

}  // namespace kore
