// Rollout-engine kernels for sm_100a:
//   * kv_append:     write new tokens' K/V (already normalised and rotated) into
//                    the paged KV cache through each sequence's block table
//   * paged_attn:    causal GQA attention of the newest q_len tokens of each
//                    sequence over its paged KV history (decode when q_len == 1,
//                    chunked "extend" prefill otherwise), split over the KV
//                    length (flash-decoding) with an in-kernel online softmax
//   * paged_combine: merges the per-split partial results
//   * sample_tokens: temperature / top-p sampling with the Gumbel-max trick
//                    (no sort: the nucleus threshold is found by bisection on
//                    probability mass), returns the token and its log-prob
// Decode attention is memory-bound (5 FLOP/byte for GQA 5:1), so it runs on
// the CUDA cores with 16-byte vector loads; the GEMMs around it use tcgen05.
//
// Reference parity: the reference samples with HF generate on a dense cache
// (kore/policy/grpo.py:2421-2425, temperature/top_p from
// kore/policy/configs.py:247-248); paging and split-KV are new here.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace dec {

constexpr int D = 128;

// new_kv: [T, 2, Hkv, D] given as separate k [T, Hkv, D] / v [T, Hkv, D] views.
// slot[t] = page * page_size + offset (precomputed on host side of the engine).
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ k, int ldk,
                                 const __nv_bfloat16* __restrict__ v, int ldv,
                                 const int* __restrict__ slots, __nv_bfloat16* __restrict__ kc,
                                 __nv_bfloat16* __restrict__ vc, int T, int Hkv) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8 elements
  const long per_tok = (long)Hkv * D / 8;
  if (i >= (long)T * per_tok) return;
  const long t = i / per_tok;
  const int r = (int)(i % per_tok) * 8;
  const long dst = (long)slots[t] * Hkv * D + r;
  *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + t * ldk + r);
  *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + t * ldv + r);
}

struct AttnParams {
  const __nv_bfloat16* q;  // [Tq, Hq, D] (row stride ldq)
  int ldq;
  const __nv_bfloat16* kc;  // [pages * page_size, Hkv, D]
  const __nv_bfloat16* vc;
  const int* block_table;   // [nseq, max_pages]
  int max_pages;
  const int* seq_lens;      // [nseq] total tokens in cache (including the new ones)
  const int* q_start;       // [nseq + 1] offsets of each sequence's query rows
  int page_size;
  int Hq, Hkv;
  float scale_log2;
  int nsplit;
  float* part_o;    // [nsplit, Tq, Hq, D]
  float* part_ml;   // [nsplit, Tq, Hq, 2] (max, sum) in log2 domain
  __nv_bfloat16* out;  // [Tq, Hq, D]
};

constexpr int kGroupMax = 8;  // q heads per kv head handled by one CTA
constexpr int kWarps = 4;

// grid: (nseq * max_q_len, Hkv, nsplit); block: 128 threads. One CTA handles
// ONE query token of one sequence and all G query heads of one kv head over
// one split of the key range.
__global__ void __launch_bounds__(kWarps * 32) paged_attn_kernel(AttnParams p, int max_q) {
  const int seq = blockIdx.x / max_q;
  const int qi = blockIdx.x % max_q;
  const int kvh = blockIdx.y;
  const int split = blockIdx.z;
  const int q0 = p.q_start[seq], q1 = p.q_start[seq + 1];
  const int qlen = q1 - q0;
  if (qi >= qlen) return;
  const int L = p.seq_lens[seq];
  const int qpos = L - qlen + qi;      // absolute position of this query token
  const int nkeys = qpos + 1;          // causal: keys 0..qpos
  const int per = (nkeys + p.nsplit - 1) / p.nsplit;
  const int k_begin = split * per;
  const int k_end = min(nkeys, k_begin + per);
  const int G = p.Hq / p.Hkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int trow = q0 + qi;

  float qv[kGroupMax][4];
#pragma unroll
  for (int g = 0; g < kGroupMax; ++g) {
    if (g < G) {
      const __nv_bfloat16* qp = p.q + (size_t)trow * p.ldq + (kvh * G + g) * D + lane * 4;
      uint2 u = *reinterpret_cast<const uint2*>(qp);
      float2 a = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
      float2 b = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
      qv[g][0] = a.x * p.scale_log2; qv[g][1] = a.y * p.scale_log2;
      qv[g][2] = b.x * p.scale_log2; qv[g][3] = b.y * p.scale_log2;
    }
  }
  float m[kGroupMax], l[kGroupMax], acc[kGroupMax][4];
#pragma unroll
  for (int g = 0; g < kGroupMax; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
    acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  }
  const int* bt = p.block_table + (size_t)seq * p.max_pages;
  for (int key = k_begin + warp; key < k_end; key += kWarps) {
    const int page = bt[key / p.page_size];
    const size_t row = ((size_t)page * p.page_size + key % p.page_size) * p.Hkv + kvh;
    uint2 ku = *reinterpret_cast<const uint2*>(p.kc + row * D + lane * 4);
    uint2 vu = *reinterpret_cast<const uint2*>(p.vc + row * D + lane * 4);
    float2 ka = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&ku.x));
    float2 kb = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&ku.y));
    float2 va = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&vu.x));
    float2 vb = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&vu.y));
    float s[kGroupMax];
#pragma unroll
    for (int g = 0; g < kGroupMax; ++g)
      s[g] = g < G ? qv[g][0] * ka.x + qv[g][1] * ka.y + qv[g][2] * kb.x + qv[g][3] * kb.y : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int g = 0; g < kGroupMax; ++g) s[g] += __shfl_xor_sync(0xffffffff, s[g], o);
#pragma unroll
    for (int g = 0; g < kGroupMax; ++g) {
      if (g >= G) continue;
      const float mn = fmaxf(m[g], s[g]);
      const float c = exp2f(m[g] - mn);
      const float e = exp2f(s[g] - mn);
      l[g] = l[g] * c + e;
      acc[g][0] = acc[g][0] * c + e * va.x;
      acc[g][1] = acc[g][1] * c + e * va.y;
      acc[g][2] = acc[g][2] * c + e * vb.x;
      acc[g][3] = acc[g][3] * c + e * vb.y;
      m[g] = mn;
    }
  }
  // combine the 4 warps through shared memory
  __shared__ float sm_m[kWarps][kGroupMax], sm_l[kWarps][kGroupMax];
  __shared__ float sm_acc[kWarps][kGroupMax][D];
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < kGroupMax; ++g) { sm_m[warp][g] = m[g]; sm_l[warp][g] = l[g]; }
  }
#pragma unroll
  for (int g = 0; g < kGroupMax; ++g)
#pragma unroll
    for (int e = 0; e < 4; ++e) sm_acc[warp][g][lane * 4 + e] = acc[g][e];
  __syncthreads();
  // thread t handles (g, d) pairs
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, sm_m[w][g]);
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      if (sm_m[w][g] == -INFINITY) continue;
      const float c = exp2f(sm_m[w][g] - mm);
      ll += sm_l[w][g] * c;
      aa += sm_acc[w][g][d] * c;
    }
    const int h = kvh * G + g;
    if (p.nsplit == 1) {
      p.out[((size_t)trow * p.Hq + h) * D + d] = __float2bfloat16(ll > 0.f ? aa / ll : 0.f);
    } else {
      const size_t tq = (size_t)p.q_start[gridDim.x / max_q];  // total query rows
      const size_t o = (((size_t)split * tq + trow) * p.Hq + h);
      p.part_o[o * D + d] = aa;
      if (d == 0) {
        p.part_ml[o * 2 + 0] = mm;
        p.part_ml[o * 2 + 1] = ll;
      }
    }
  }
}

// Decode (one query token per sequence), key-per-lane layout: every lane of a
// warp owns one key of a 32-key chunk, reads that key's whole 256-byte K row
// and scores it against the G query heads kept in shared memory, so the
// softmax needs one warp max per chunk instead of a shuffle tree per key. The
// P.V product then walks the chunk's V rows with lanes spread over D (coalesced
// 256-byte rows). 32-key chunks never cross a page (page_size % 32 == 0).
// Partial results use the layout of paged_attn_kernel, so paged_combine_kernel
// merges the splits.
template <int G>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_kernel(AttnParams p) {
  const int seq = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int trow = p.q_start[seq];
  const int nkeys = p.seq_lens[seq];
  const int per = ((nkeys + p.nsplit - 1) / p.nsplit + 31) & ~31;
  const int k_begin = split * per;
  const int k_end = min(nkeys, k_begin + per);
  __shared__ __align__(16) float sq[G][D];
  __shared__ float sp[kWarps][G][32];
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    sq[g][d] = __bfloat162float(p.q[(size_t)trow * p.ldq + (kvh * G + g) * D + d]) * p.scale_log2;
  }
  __syncthreads();
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY; l[g] = 0.f;
    acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.f;
  }
  const int* bt = p.block_table + (size_t)seq * p.max_pages;
  const size_t hstride = (size_t)p.Hkv * D;
  for (int c = k_begin + warp * 32; c < k_end; c += kWarps * 32) {
    const int page = bt[c / p.page_size];
    const size_t base = ((size_t)page * p.page_size + c % p.page_size) * hstride + (size_t)kvh * D;
    const int key = c + lane;
    const bool valid = key < k_end;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
    if (valid) {
      const uint4* kr = reinterpret_cast<const uint4*>(p.kc + base + (size_t)lane * hstride);
#pragma unroll 4
      for (int j = 0; j < D / 8; ++j) {
        const uint4 u = kr[j];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
        const float2 k0 = __bfloat1622float2(h[0]), k1 = __bfloat1622float2(h[1]);
        const float2 k2 = __bfloat1622float2(h[2]), k3 = __bfloat1622float2(h[3]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float4 qa = *reinterpret_cast<const float4*>(&sq[g][j * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&sq[g][j * 8 + 4]);
          s[g] += qa.x * k0.x + qa.y * k0.y + qa.z * k1.x + qa.w * k1.y +
                  qb.x * k2.x + qb.y * k2.y + qb.z * k3.x + qb.w * k3.y;
        }
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float cm = valid ? s[g] : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffff, cm, o));
      const float mn = fmaxf(m[g], cm);
      const float corr = exp2f(m[g] - mn);
      const float e = valid ? exp2f(s[g] - mn) : 0.f;
      l[g] = l[g] * corr + e;                 // per-lane partial of the row sum
      acc[g][0] *= corr; acc[g][1] *= corr; acc[g][2] *= corr; acc[g][3] *= corr;
      m[g] = mn;
      sp[warp][g][lane] = e;
    }
    __syncwarp();
    const int nk = min(32, k_end - c);
    const __nv_bfloat16* vr = p.vc + base + lane * 4;
#pragma unroll 8
    for (int kk = 0; kk < nk; ++kk) {
      const uint2 vu = *reinterpret_cast<const uint2*>(vr + (size_t)kk * hstride);
      const float2 va = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vu.x));
      const float2 vb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vu.y));
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pe = sp[warp][g][kk];
        acc[g][0] += pe * va.x; acc[g][1] += pe * va.y; acc[g][2] += pe * vb.x; acc[g][3] += pe * vb.y;
      }
    }
    __syncwarp();
  }
  // row sums across lanes, then merge the warps through shared memory
  __shared__ float sm_m[kWarps][G], sm_l[kWarps][G];
  __shared__ float sm_acc[kWarps][G][D];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float t = l[g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffff, t, o);
    if (lane == 0) { sm_m[warp][g] = m[g]; sm_l[warp][g] = t; }
#pragma unroll
    for (int e = 0; e < 4; ++e) sm_acc[warp][g][lane * 4 + e] = acc[g][e];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, sm_m[w][g]);
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      if (sm_m[w][g] == -INFINITY) continue;
      const float c = exp2f(sm_m[w][g] - mm);
      ll += sm_l[w][g] * c;
      aa += sm_acc[w][g][d] * c;
    }
    const int h = kvh * G + g;
    if (p.nsplit == 1) {
      p.out[((size_t)trow * p.Hq + h) * D + d] = __float2bfloat16(ll > 0.f ? aa / ll : 0.f);
    } else {
      const size_t tq = (size_t)p.q_start[gridDim.x];
      const size_t o = ((size_t)split * tq + trow) * p.Hq + h;
      p.part_o[o * D + d] = aa;
      if (d == 0) {
        p.part_ml[o * 2 + 0] = mm;
        p.part_ml[o * 2 + 1] = ll;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Decode attention with a TMA pipeline (one query token per sequence).
// CTA = (sequence, kv head, split); warp 0 streams the split's pages of this
// kv head's K and V through a STAGES-deep ring of shared-memory buffers with
// plain (non-multicast) TMA tile loads (one 64-key page per stage, two 64-column
// boxes per matrix so the 128-byte swizzle applies); warps 1..4 consume a page
// together, 16 keys each, on mma.sync tensor-core fragments: the G query heads
// are the rows of one 16-row A operand (rows G..15 zero), K fragments come from
// ldmatrix on the swizzled tile (16-byte chunk c of row r sits at chunk c ^ (r % 8)),
// V fragments from ldmatrix.trans, and P moves from the score accumulators into
// the A operand of P.V without leaving registers. Decode attention is bound by
// HBM; the tensor-core fragments only keep the instruction count far below the
// bytes the TMA ring delivers. Two CTAs fit an SM.
constexpr int kTmaStages = 3;
constexpr int kPage = 64;                          // keys per stage (= cache page size)
constexpr int kStageK = kPage * D * 2;             // 16 KB of K per stage
constexpr int kConsumers = 4;
constexpr int kKeysPerWarp = kPage / kConsumers;   // 16
constexpr int kTmaThreads = 32 * (1 + kConsumers);

struct TmaDecodeSmem {
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = kTmaStages * kStageK;
  static constexpr int BAR_OFF = 2 * kTmaStages * kStageK;
  static constexpr int TOTAL = BAR_OFF + 64 + 1024;
};

template <int G>
__global__ void __launch_bounds__(kTmaThreads) paged_decode_tma_kernel(
    const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  extern __shared__ __align__(1024) uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + TmaDecodeSmem::BAR_OFF);
  uint64_t* empty = full + kTmaStages;
  __shared__ __align__(16) float sq[G][D];
  __shared__ float sm_m[kConsumers][G], sm_l[kConsumers][G];
  __shared__ int s_abort;
  // the merge buffer reuses the K stages once every page has been consumed
  float (*sm_acc)[G][D] = reinterpret_cast<float (*)[G][D]>(dsm + TmaDecodeSmem::K_OFF);
  static_assert(kConsumers * G * D * 4 <= kTmaStages * kStageK, "merge buffer fits the K stages");

  const int seq = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int trow = p.q_start[seq];
  const int nkeys = p.seq_lens[seq];
  const int npages = (nkeys + kPage - 1) / kPage;
  const int per = (npages + p.nsplit - 1) / p.nsplit;       // pages per split
  const int pg0 = split * per, pg1 = min(npages, pg0 + per);
  const int* bt = p.block_table + (size_t)seq * p.max_pages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTmaStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    s_abort = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    sq[g][d] = __bfloat162float(p.q[(size_t)trow * p.ldq + (kvh * G + g) * D + d]) * p.scale_log2;
  }
  __syncthreads();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int pg = pg0; pg < pg1; ++pg) {
        if (!mbar_wait(&empty[stage], phase ^ 1)) { s_abort = 1; break; }
        const int y = bt[pg] * kPage;
        uint8_t* kb = dsm + TmaDecodeSmem::K_OFF + stage * kStageK;
        uint8_t* vb = dsm + TmaDecodeSmem::V_OFF + stage * kStageK;
        mbar_arrive_expect_tx(&full[stage], 2 * kStageK);
        tma_load_2d(kb, &tmK, &full[stage], kvh * D, y);
        tma_load_2d(kb + kStageK / 2, &tmK, &full[stage], kvh * D + 64, y);
        tma_load_2d(vb, &tmV, &full[stage], kvh * D, y);
        tma_load_2d(vb + kStageK / 2, &tmV, &full[stage], kvh * D + 64, y);
        if (++stage == kTmaStages) { stage = 0; phase ^= 1; }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- consumers (mma.sync)
    // Per page each warp owns 16 keys. S[16 x 16] = Q[16 x 128] K^T with the G
    // query heads in rows 0..G-1 (rows G..15 zero), then O[16 x 128] += P V. The
    // K fragments come from ldmatrix on the swizzled tile, the V fragments from
    // ldmatrix.trans; P goes from the S accumulators straight into A fragments.
    const int cw = warp - 1;
    const int gid = lane >> 2, tig = lane & 3;
    uint32_t qa[8][4];                          // Q A-fragments, 8 k-steps of 16 dims
    {
      const bool hv = gid < G;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int d0 = kk * 16 + 2 * tig;
        qa[kk][0] = hv ? pack_bf16(sq[gid][d0], sq[gid][d0 + 1]) : 0u;
        qa[kk][1] = 0u;                          // rows 8..15: padding
        qa[kk][2] = hv ? pack_bf16(sq[gid][d0 + 8], sq[gid][d0 + 9]) : 0u;
        qa[kk][3] = 0u;
      }
    }
    float o[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    float mrow = -INFINITY, lrow = 0.f;          // softmax state of head `gid` (replicated in the quad)
    int stage = 0;
    uint32_t phase = 0;
    const uint32_t kbase0 = smem_u32(dsm + TmaDecodeSmem::K_OFF);
    const uint32_t vbase0 = smem_u32(dsm + TmaDecodeSmem::V_OFF);
    for (int pg = pg0; pg < pg1 && !s_abort; ++pg) {
      if (!mbar_wait(&full[stage], phase)) { s_abort = 1; break; }
      const uint32_t kb = kbase0 + stage * kStageK;
      const uint32_t vb = vbase0 + stage * kStageK;
      const int key0 = cw * kKeysPerWarp;        // first key of this warp in the page
      // ---- scores: two n8 tiles (keys key0..+7, key0+8..+15)
      float sc[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t) sc[t][0] = sc[t][1] = sc[t][2] = sc[t][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {           // pairs of k-steps: 32 dims per ldmatrix.x4
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int mi = lane >> 3, r = lane & 7;
          const int row = key0 + t * 8 + r;
          const int d = kp * 32 + mi * 8;       // 8-dim chunk this lane addresses
          const uint32_t addr = kb + (d >> 6) * (kStageK / 2) + row * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4);
          uint32_t b0, b1, b2, b3;
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                       : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(addr));
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t* A = qa[2 * kp + h];
            const uint32_t bb0 = h == 0 ? b0 : b2, bb1 = h == 0 ? b1 : b3;
            asm volatile(
                "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                "{%0,%1,%2,%3};"
                : "+f"(sc[t][0]), "+f"(sc[t][1]), "+f"(sc[t][2]), "+f"(sc[t][3])
                : "r"(A[0]), "r"(A[1]), "r"(A[2]), "r"(A[3]), "r"(bb0), "r"(bb1));
          }
        }
      }
      // ---- online softmax of row gid over this warp's 16 keys (4 values per thread)
      float v[4];
      int kv[4];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          kv[2 * t + c] = pg * kPage + key0 + t * 8 + 2 * tig + c;
          v[2 * t + c] = kv[2 * t + c] < nkeys ? sc[t][c] : -INFINITY;   // q carries the log2 scale
        }
      float mx = fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffff, mx, 2));
      const float mn = fmaxf(mrow, mx);
      const float corr = mn == -INFINITY ? 1.f : exp2f(mrow - mn);
      float e[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) e[i] = v[i] == -INFINITY ? 0.f : exp2f(v[i] - mn);
      lrow = lrow * corr + (e[0] + e[1]) + (e[2] + e[3]);
      mrow = mn;
      if (corr != 1.f) {
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) { o[nt][0] *= corr; o[nt][1] *= corr; }
      }
      // ---- O += P V: P (16 x 16 keys) as one A fragment, V via ldmatrix.trans
      uint32_t pa[4];
      pa[0] = pack_bf16(e[0], e[1]);             // row gid, keys 2tig..      (tile 0)
      pa[1] = 0u;                                 // row gid + 8: padding
      pa[2] = pack_bf16(e[2], e[3]);             // row gid, keys 8 + 2tig..  (tile 1)
      pa[3] = 0u;
#pragma unroll
      for (int np = 0; np < 8; ++np) {           // 16 dims (two n8 tiles) per ldmatrix.x4.trans
        const int mi = lane >> 3, r = lane & 7;
        const int row = key0 + (mi & 1) * 8 + r;
        const int d = np * 16 + (mi >> 1) * 8;
        const uint32_t addr = vb + (d >> 6) * (kStageK / 2) + row * 128 + ((((d & 63) >> 3) ^ (row & 7)) << 4);
        uint32_t b0, b1, b2, b3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(addr));
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(o[2 * np][0]), "+f"(o[2 * np][1]), "+f"(o[2 * np][2]), "+f"(o[2 * np][3])
            : "r"(pa[0]), "r"(pa[1]), "r"(pa[2]), "r"(pa[3]), "r"(b0), "r"(b1));
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(o[2 * np + 1][0]), "+f"(o[2 * np + 1][1]), "+f"(o[2 * np + 1][2]), "+f"(o[2 * np + 1][3])
            : "r"(pa[0]), "r"(pa[1]), "r"(pa[2]), "r"(pa[3]), "r"(b2), "r"(b3));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == kTmaStages) { stage = 0; phase ^= 1; }
    }
    // every consumer is done reading the K stages before any overwrites them
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kConsumers) : "memory");
    float lsum = lrow + __shfl_xor_sync(0xffffffff, lrow, 1);
    lsum += __shfl_xor_sync(0xffffffff, lsum, 2);
    if (gid < G) {
      if (tig == 0) { sm_m[cw][gid] = mrow; sm_l[cw][gid] = lsum; }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        sm_acc[cw][gid][nt * 8 + 2 * tig] = o[nt][0];
        sm_acc[cw][gid][nt * 8 + 2 * tig + 1] = o[nt][1];
      }
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) mm = fmaxf(mm, sm_m[w][g]);
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumers; ++w) {
      if (sm_m[w][g] == -INFINITY) continue;
      const float c = exp2f(sm_m[w][g] - mm);
      ll += sm_l[w][g] * c;
      aa += sm_acc[w][g][d] * c;
    }
    const int h = kvh * G + g;
    if (p.nsplit == 1) {
      p.out[((size_t)trow * p.Hq + h) * D + d] = __float2bfloat16(ll > 0.f ? aa / ll : 0.f);
    } else {
      const size_t tq = (size_t)p.q_start[gridDim.x];
      const size_t o = ((size_t)split * tq + trow) * p.Hq + h;
      p.part_o[o * D + d] = aa;
      if (d == 0) {
        p.part_ml[o * 2 + 0] = mm;
        p.part_ml[o * 2 + 1] = ll;
      }
    }
  }
}

__global__ void paged_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                     __nv_bfloat16* __restrict__ out, int Tq, int Hq, int nsplit) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // over Tq * Hq * D
  if (i >= (long)Tq * Hq * D) return;
  const long row = i / D;  // (t, h)
  const int d = i % D;
  float mm = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mm = fmaxf(mm, part_ml[((size_t)s * Tq * Hq + row) * 2]);
  float ll = 0.f, aa = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const size_t o = (size_t)s * Tq * Hq + row;
    const float ms = part_ml[o * 2];
    if (ms == -INFINITY) continue;
    const float c = exp2f(ms - mm);
    ll += part_ml[o * 2 + 1] * c;
    aa += part_o[o * D + d] * c;
  }
  out[row * D + d] = __float2bfloat16(ll > 0.f ? aa / ll : 0.f);
}

// ---------------------------------------------------------------- sampling
// Counter-based hash ("lowbias32", C. Wellons 2018) -> uniform in (0, 1).
KORE_DEV uint32_t hash32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}
KORE_DEV float uniform01(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t h = hash32(a ^ hash32(b ^ hash32(c)));
  return ((h >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

constexpr int kSampThreads = 1024;

template <typename T>
KORE_DEV float blk_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float w = __shfl_xor_sync(0xffffffff, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float r = is_max ? -INFINITY : 0.f;
  for (int i = 0; i < (int)(blockDim.x / 32); ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

// One CTA per row. logits [B, V] bf16. Writes token[b] and its log-prob under
// the temperature-scaled full distribution.
__global__ void __launch_bounds__(kSampThreads) sample_kernel(
    const __nv_bfloat16* __restrict__ logits, int ld, int V, float inv_temp, float top_p,
    uint32_t seed, uint32_t step, const int* __restrict__ step_ptr, int greedy, long* __restrict__ out_tok,
    float* __restrict__ out_lp) {
  if (step_ptr != nullptr) step = (uint32_t)*step_ptr;
  __shared__ float red[32];
  __shared__ float s_best[32];
  __shared__ int s_bidx[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* z = logits + (size_t)row * ld;
  // pass 1: max and sum of exp
  float mx = -INFINITY;
  for (int j = threadIdx.x; j < V; j += blockDim.x) mx = fmaxf(mx, __bfloat162float(z[j]) * inv_temp);
  mx = blk_reduce<float>(mx, red, true);
  float sum = 0.f;
  for (int j = threadIdx.x; j < V; j += blockDim.x) sum += exp2f((__bfloat162float(z[j]) * inv_temp - mx) * 1.4426950408889634f);
  sum = blk_reduce<float>(sum, red, false);
  const float lse = mx + __logf(sum);
  // nucleus threshold (in logit units): largest t with mass(z >= t) >= top_p
  float thr = -INFINITY;
  if (top_p < 1.f) {
    float lo = mx - 40.f, hi = mx;  // mass(z >= lo) ~ 1, mass(z >= hi) small
    for (int it = 0; it < 24; ++it) {
      const float mid = 0.5f * (lo + hi);
      float mass = 0.f;
      for (int j = threadIdx.x; j < V; j += blockDim.x) {
        const float zz = __bfloat162float(z[j]) * inv_temp;
        if (zz >= mid) mass += __expf(zz - lse);
      }
      mass = blk_reduce<float>(mass, red, false);
      if (mass >= top_p) lo = mid; else hi = mid;
    }
    thr = lo;
  }
  // Gumbel-max over the nucleus
  float best = -INFINITY;
  int bidx = 0;
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float zz = __bfloat162float(z[j]) * inv_temp;
    if (zz < thr) continue;
    float g = zz;
    if (!greedy) {
      const float u = uniform01(seed, step * 0x9E3779B9u + row, (uint32_t)j);
      g -= __logf(-__logf(u));
    }
    if (g > best) { best = g; bidx = j; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float b2 = __shfl_xor_sync(0xffffffff, best, o);
    int i2 = __shfl_xor_sync(0xffffffff, bidx, o);
    if (b2 > best || (b2 == best && i2 < bidx)) { best = b2; bidx = i2; }
  }
  const int wid = threadIdx.x / 32, lane = threadIdx.x & 31;
  if (lane == 0) { s_best[wid] = best; s_bidx[wid] = bidx; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float bb = -INFINITY;
    int bi = 0;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i)
      if (s_best[i] > bb || (s_best[i] == bb && s_bidx[i] < bi)) { bb = s_best[i]; bi = s_bidx[i]; }
    out_tok[row] = bi;
    out_lp[row] = __bfloat162float(z[bi]) * inv_temp - lse;
  }
}

}  // namespace dec

void kv_append(const at::Tensor& k, const at::Tensor& v, const at::Tensor& slots, at::Tensor& kc,
               at::Tensor& vc) {
  using namespace dec;
  const int T = k.size(0), Hkv = k.size(1);
  TORCH_CHECK(k.size(2) == D && v.size(2) == D && k.stride(2) == 1 && k.stride(1) == D &&
                  v.stride(1) == D, "kv_append: expected [T, Hkv, 128] views with contiguous heads");
  TORCH_CHECK(slots.scalar_type() == at::kInt && slots.numel() == T, "slots int32 [T]");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(k.device());
  const long n = (long)T * Hkv * D / 8;
  kv_append_kernel<<<(int)((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)k.data_ptr(), k.stride(0), (const __nv_bfloat16*)v.data_ptr(), v.stride(0),
      slots.data_ptr<int>(), (__nv_bfloat16*)kc.data_ptr(), (__nv_bfloat16*)vc.data_ptr(), T, Hkv);
  check_cuda(cudaGetLastError(), "kv_append");
}

// q: [Tq, Hq, 128] (row stride); caches [slots, Hkv, 128]; returns out [Tq, Hq, 128].
void paged_attention(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc,
                     const at::Tensor& block_table, const at::Tensor& seq_lens,
                     const at::Tensor& q_start, int64_t max_q, int64_t page_size, double scale,
                     int64_t nsplit, at::Tensor& out, const c10::optional<at::Tensor>& part_o,
                     const c10::optional<at::Tensor>& part_ml) {
  using namespace dec;
  const int Tq = q.size(0), Hq = q.size(1), Hkv = kc.size(1);
  TORCH_CHECK(q.size(2) == D && q.stride(2) == 1 && q.stride(1) == D, "q layout");
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= kGroupMax, "GQA group too large");
  const int nseq = seq_lens.numel();
  if (Tq == 0 || nseq == 0) return;
  if (nsplit > 1)
    TORCH_CHECK(part_o.has_value() && part_ml.has_value() &&
                    part_o->numel() >= (int64_t)nsplit * Tq * Hq * D && part_ml->numel() >= (int64_t)nsplit * Tq * Hq * 2,
                "split-KV needs partial buffers");
  c10::cuda::CUDAGuard g(q.device());
  AttnParams p;
  p.q = (const __nv_bfloat16*)q.data_ptr();
  p.ldq = q.stride(0);
  p.kc = (const __nv_bfloat16*)kc.data_ptr();
  p.vc = (const __nv_bfloat16*)vc.data_ptr();
  p.block_table = block_table.data_ptr<int>();
  p.max_pages = block_table.size(1);
  p.seq_lens = seq_lens.data_ptr<int>();
  p.q_start = q_start.data_ptr<int>();
  p.page_size = page_size;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = (float)scale * 1.4426950408889634f;
  p.nsplit = nsplit;
  p.part_o = nsplit > 1 ? part_o->data_ptr<float>() : nullptr;
  p.part_ml = nsplit > 1 ? part_ml->data_ptr<float>() : nullptr;
  p.out = (__nv_bfloat16*)out.data_ptr();
  auto st = at::cuda::getCurrentCUDAStream();
  const int G = Hq / Hkv;
  if (max_q == 1 && page_size == kPage && Tq == nseq && (G == 1 || G == 2 || G == 4 || G == 5 || G == 8)) {
    // TMA-pipelined decode: tensor maps over the caches viewed as [slots, Hkv * 128]
    auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint64_t slots = (uint64_t)kc.size(0);
    CUtensorMap tk = make_tmap_2d(kc.data_ptr(), bf, 2, (uint64_t)Hkv * D, slots, (uint64_t)Hkv * D, 64, kPage);
    CUtensorMap tv = make_tmap_2d(vc.data_ptr(), bf, 2, (uint64_t)Hkv * D, slots, (uint64_t)Hkv * D, 64, kPage);
    dim3 grid(nseq, Hkv, nsplit);
    const int smem = TmaDecodeSmem::TOTAL;
    static bool attr[64][9] = {};
    int dev = 0;
    check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
#define KORE_DEC_TMA(GG)                                                                                   \
  {                                                                                                        \
    auto kfn = paged_decode_tma_kernel<GG>;                                                                \
    if (!attr[dev][GG]) {                                                                                  \
      check_cuda(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "decode smem"); \
      attr[dev][GG] = true;                                                                                \
    }                                                                                                      \
    kfn<<<grid, kTmaThreads, smem, st>>>(tk, tv, p);                                                       \
  }
    switch (G) {
      case 1: KORE_DEC_TMA(1) break;
      case 2: KORE_DEC_TMA(2) break;
      case 4: KORE_DEC_TMA(4) break;
      case 5: KORE_DEC_TMA(5) break;
      default: KORE_DEC_TMA(8) break;
    }
#undef KORE_DEC_TMA
    check_cuda(cudaGetLastError(), "paged_decode_tma");
  } else if (max_q == 1 && page_size % 32 == 0 && Tq == nseq) {
    dim3 grid(nseq, Hkv, nsplit);
    switch (G) {
      case 1: paged_decode_kernel<1><<<grid, kWarps * 32, 0, st>>>(p); break;
      case 2: paged_decode_kernel<2><<<grid, kWarps * 32, 0, st>>>(p); break;
      case 4: paged_decode_kernel<4><<<grid, kWarps * 32, 0, st>>>(p); break;
      case 5: paged_decode_kernel<5><<<grid, kWarps * 32, 0, st>>>(p); break;
      case 8: paged_decode_kernel<8><<<grid, kWarps * 32, 0, st>>>(p); break;
      default: paged_attn_kernel<<<dim3(nseq, Hkv, nsplit), kWarps * 32, 0, st>>>(p, 1);
    }
    check_cuda(cudaGetLastError(), "paged_decode");
  } else {
    dim3 grid(nseq * max_q, Hkv, nsplit);
    paged_attn_kernel<<<grid, kWarps * 32, 0, st>>>(p, (int)max_q);
    check_cuda(cudaGetLastError(), "paged_attn");
  }
  if (nsplit > 1) {
    const long n = (long)Tq * Hq * D;
    paged_combine_kernel<<<(int)((n + 255) / 256), 256, 0, st>>>(p.part_o, p.part_ml, p.out, Tq, Hq, nsplit);
    check_cuda(cudaGetLastError(), "paged_combine");
  }
}

void sample_tokens(const at::Tensor& logits, double temperature, double top_p, int64_t seed,
                   int64_t step, at::Tensor& tokens, at::Tensor& logprobs,
                   const c10::optional<at::Tensor>& step_dev) {
  using namespace dec;
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "logits bf16 rows");
  const int B = logits.size(0), V = logits.size(1);
  if (B == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  const bool greedy = temperature <= 0.0;
  sample_kernel<<<B, kSampThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      (const __nv_bfloat16*)logits.data_ptr(), logits.stride(0), V,
      greedy ? 1.f : (float)(1.0 / temperature), greedy ? 1.f : (float)top_p, (uint32_t)seed,
      (uint32_t)step, step_dev ? step_dev->data_ptr<int>() : nullptr, greedy ? 1 : 0, tokens.data_ptr<long>(),
      logprobs.data_ptr<float>());
  check_cuda(cudaGetLastError(), "sample_tokens");
}

}  // namespace kore
