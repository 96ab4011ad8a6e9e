// Causal GQA flash attention for sm_100a (head_dim 128), packed varlen
// sequences, forward and backward, on tcgen05 tensor cores.
//
// Forward (one CTA per (128-row query block, query head)):
//   warp 0      TMA producer: Q once, then K_j / V_j tiles (2-stage rings)
//   warp 1      MMA issuer:   S_{j+1} = Q K_{j+1}^T (TMEM, ping-pong) is issued
//                             before O += P_j V_j, so the next score tile is
//                             computed while the softmax warps work on this one
//   warps 2..5  softmax: one query row per thread read from TMEM, online
//               max/sum in the log2 domain, P (bf16) written to shared memory
//               in the 128B-swizzled K-major layout UMMA reads; O in TMEM is
//               only rescaled when the running max grows by more than 2^8
//               (lazy rescaling; only then does a softmax warp wait for the
//               previous PV product), then normalised in the epilogue.
// Backward (one CTA per (128-row key block, kv head)): loops over the query
//   heads of the GQA group and the causal query blocks, recomputing
//   S^T = K Q^T, P^T = exp(S^T - lse), dP^T = V dO^T, dS^T = P^T (dP^T - delta)
//   with dV += P^T dO and dK += dS^T Q accumulated in TMEM for the whole CTA,
//   and dQ partials (dS K) added to an fp32 scratch accumulator in global
//   memory with vector atomics; a final kernel converts it to bf16.
//
// Reference parity: the reference runs attention through SDPA /
// flash_attention_2 inside HF (kore/policy/configs.py:682-700).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace attn {

constexpr int D = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int kThreads = 192;
constexpr int TILE_BYTES = 128 * D * 2;  // 32 KB: 128 rows x 128 bf16 as two 64-col swizzle atoms
constexpr float kLog2e = 1.4426950408889634f;

KORE_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  const uint32_t (&a)[16] = *reinterpret_cast<const uint32_t(*)[16]>(&r[0]);
  const uint32_t (&b)[16] = *reinterpret_cast<const uint32_t(*)[16]>(&r[16]);
  tmem_st16(taddr, a);
  tmem_st16(taddr + 16, b);
}

// Descriptor of a 128-row, 128-column bf16 tile stored as two K-major
// 64-column SW128 atoms (16 KB apart), advanced to K-step kk (16 columns).
KORE_DEV uint64_t kmajor_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
// Same tile read as an MN-major operand (rows = K, the 128 columns = N in two
// 64-wide blocks 16 KB apart), advanced to K-step kk (16 rows).
KORE_DEV uint64_t mnmajor_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + kk * 2048, 16384, 1024);
}

struct FwdParams {
  const int* cu_seqlens;
  int nseq;
  int nqblk;  // blocks per sequence slot (ceil(max_seqlen / 128))
  int Hq, Hkv;
  float scale_log2;
  __nv_bfloat16* o;  // [T, Hq, D]
  float* lse;        // [Hq, T] natural log
  int T;
};

// 64-row, 128-column tile (two 8 KB atoms): K-major operand at K-step kk.
KORE_DEV uint64_t kmajor64_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
}
// Same 64-row tile as an MN-major operand (rows = K, N = 128 in two 64-wide
// blocks 8 KB apart) at K-step kk.
KORE_DEV uint64_t mnmajor64_desc(uint32_t base, int kk) { return make_sw128_desc(base + kk * 2048, 8192, 1024); }
// 128-row x 64-column tile (one atom): K-major at K-step kk / MN-major (N = 64) at K-step kk.
KORE_DEV uint64_t kmajor_narrow_desc(uint32_t base, int kk) { return make_sw128_desc(base + kk * 32, 16, 1024); }
KORE_DEV uint64_t mnmajor_narrow_desc(uint32_t base, int kk) { return make_sw128_desc(base + kk * 2048, 16384, 1024); }

// Forward tiling: 128 query rows x 64-key blocks. P lives in TMEM (aliasing
// its S buffer) and feeds the PV product as the TMEM operand. Shared memory
// (Q + two K and two V stages, 96 KB) and TMEM (two 64-column S buffers +
// 128-column O = 256 columns) are sized so that two CTAs share an SM: while
// one CTA's softmax warps work, the other's products keep the tensor pipe busy.
constexpr int FBKV = 64;
constexpr int KV_TILE_BYTES = FBKV * D * 2;   // 16 KB: 64 rows as two 8 KB swizzle atoms
constexpr int kFwdStages = 2;
constexpr int kFwdTmemCols = 256;
struct FwdSmem {
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = TILE_BYTES;                          // kFwdStages stages
  static constexpr int V_OFF = K_OFF + kFwdStages * KV_TILE_BYTES;  // kFwdStages stages
  static constexpr int BAR_OFF = V_OFF + kFwdStages * KV_TILE_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
};
static_assert(2 * (FwdSmem::TOTAL + 1024) <= 228 * 1024, "fwd smem: two CTAs per SM");

__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, FwdParams p) {
  using S = FwdSmem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [kFwdStages]
  uint64_t* k_empty = bars + 3;   // [kFwdStages]
  uint64_t* v_full = bars + 5;    // [kFwdStages]
  uint64_t* v_empty = bars + 7;   // [kFwdStages]
  uint64_t* s_full = bars + 9;    // [2]
  uint64_t* p_full = bars + 11;   // [2]
  uint64_t* o_done = bars + 13;   // one phase per PV product
  uint64_t* o_final = bars + 14;  // the last PV product
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // ---- work item: longest (latest) query blocks first
  const int slot = p.nseq * p.nqblk - 1 - blockIdx.x;
  const int seq = slot / p.nqblk;
  const int qb = slot % p.nqblk;
  const int h = blockIdx.y;
  const int kvh = h / (p.Hq / p.Hkv);
  const int s0 = p.cu_seqlens[seq];
  const int len = p.cu_seqlens[seq + 1] - s0;
  const int q0 = qb * BQ;
  if (q0 >= len) return;  // whole CTA exits before any barrier / TMEM use
  const int nkv = (min(q0 + BQ, len) + FBKV - 1) / FBKV;   // causal: key blocks up to the last query row
  const int warp = threadIdx.x / 32;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kFwdStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kFwdTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: [0,64) S/P buffer 0, [64,128) S/P buffer 1, [128,256) O
  constexpr uint32_t T_O = 128;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(smem + S::Q_OFF, &tmQ, q_full, h * D, s0 + q0);
      tma_load_2d(smem + S::Q_OFF + 16384, &tmQ, q_full, h * D + 64, s0 + q0);
      for (int j = 0; j < nkv && !*abort_flag; ++j) {
        const int st = j % kFwdStages;
        const uint32_t ph = (j / kFwdStages) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1)) { *abort_flag = 1; break; }
        uint8_t* kt = smem + S::K_OFF + st * KV_TILE_BYTES;
        mbar_arrive_expect_tx(&k_full[st], KV_TILE_BYTES);
        tma_load_2d(kt, &tmK, &k_full[st], kvh * D, s0 + j * FBKV);
        tma_load_2d(kt + 8192, &tmK, &k_full[st], kvh * D + 64, s0 + j * FBKV);
        if (!mbar_wait(&v_empty[st], ph ^ 1)) { *abort_flag = 1; break; }
        uint8_t* vt = smem + S::V_OFF + st * KV_TILE_BYTES;
        mbar_arrive_expect_tx(&v_full[st], KV_TILE_BYTES);
        tma_load_2d(vt, &tmV, &v_full[st], kvh * D, s0 + j * FBKV);
        tma_load_2d(vt + 8192, &tmV, &v_full[st], kvh * D + 64, s0 + j * FBKV);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t idesc_qk = make_idesc_bf16(BQ, FBKV, false, false);
    constexpr uint32_t idesc_pv = make_idesc_bf16(BQ, D, false, true);   // A = P from TMEM (K-major)
    if (elect_one()) {
      const uint32_t qa = smem_u32(smem + S::Q_OFF);
      bool ok = mbar_wait(q_full, 0);
      auto issue_s = [&](int j) -> bool {
        const int ks = j % kFwdStages;
        if (!mbar_wait(&k_full[ks], (j / kFwdStages) & 1)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + S::K_OFF + ks * KV_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16_ss(tmem + (j & 1) * FBKV, kmajor_desc(qa, kk), kmajor64_desc(ka, kk), idesc_qk, kk > 0);
        umma_commit(&k_empty[ks]);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkv && ok; ++j) {
        // S_{j+1} goes into the buffer whose P_{j-1} the already-issued PV_{j-1} reads (in-order pipe)
        if (j + 1 < nkv && !issue_s(j + 1)) { ok = false; break; }
        const int st = j & 1;
        const int vs = j % kFwdStages;
        if (!mbar_wait(&p_full[st], (j >> 1) & 1)) { ok = false; break; }
        if (!mbar_wait(&v_full[vs], (j / kFwdStages) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t va = smem_u32(smem + S::V_OFF + vs * KV_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < FBKV / 16; ++kk)   // P_j: 32 TMEM columns of packed bf16 pairs, 8 per K-step
          umma_f16_ts(tmem + T_O, tmem + st * FBKV + kk * 8, mnmajor64_desc(va, kk), idesc_pv,
                      (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&v_empty[vs]);
        umma_commit(o_done);
      }
      if (ok) umma_commit(o_final);
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- softmax warps
    const int q = warp & 3;
    const int lane = threadIdx.x & 31;
    const int row = q * 32 + lane;  // row within the query block
    const int qi = q0 + row;        // query position within the sequence
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float m = -INFINITY, l = 0.f;
    float sv[FBKV];
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1)) { ok = false; break; }
      tc_fence_after();
      {
        uint32_t r[2][32];
        tmem_ld32(tmem + lane_base + st * FBKV, r[0]);
        tmem_ld32(tmem + lane_base + st * FBKV + 32, r[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(r[c][i]);   // raw scores
      }
      const int kv0 = j * FBKV;
      const bool edge = (kv0 + FBKV > q0) || (kv0 + FBKV > len);
      if (edge) {
#pragma unroll
        for (int i = 0; i < FBKV; ++i)
          if (kv0 + i > qi || kv0 + i >= len) sv[i] = -INFINITY;
      }
      // row max of the raw scores (the log2 scale is positive, so it commutes)
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int i = 0; i < FBKV; i += 8) {
        mx4[0] = fmax3f(mx4[0], sv[i], sv[i + 1]);
        mx4[1] = fmax3f(mx4[1], sv[i + 2], sv[i + 3]);
        mx4[2] = fmax3f(mx4[2], sv[i + 4], sv[i + 5]);
        mx4[3] = fmax3f(mx4[3], sv[i + 6], sv[i + 7]);
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      float m_new = fmaxf(m, mx);
      const bool need = (m == -INFINITY) ? true : (m_new > m + 8.f);
      if (j > 0) {
        // O is touched only when a row's max grew past the lazy threshold; only
        // then wait for PV_{j-1}. Parity waits on o_done are unambiguous here:
        // S_j's commit implies PV_{j-2} is done and PV_j is not yet issued, so
        // o_done has completed j-1 or j phases.
        const float alpha = need ? exp2f(m - m_new) : 1.f;
        if (__any_sync(0xffffffff, need && m != -INFINITY)) {
          if (!mbar_wait(o_done, (j - 1) & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            const uint32_t a = tmem + lane_base + T_O + c * 32;
            tmem_ld32(a, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tmem_st32(a, r);
          }
          tmem_wait_st();
        }
        if (need) l *= alpha;
      }
      if (need) m = m_new;
      const float mref = (m == -INFINITY) ? 0.f : m;
      // p = 2^(s * scale_log2 - m): one packed FMA per two scores, packed row sums
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
      const uint64_t nm2 = f2_pack(-mref, -mref);
      uint64_t rs2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < FBKV; i += 2) {
        float a, b;
        f2_unpack(f2_fma(f2_pack(sv[i], sv[i + 1]), sc2, nm2), a, b);
        sv[i] = exp2f(a);
        sv[i + 1] = exp2f(b);
        rs2[(i >> 1) & 1] = f2_add(rs2[(i >> 1) & 1], f2_pack(sv[i], sv[i + 1]));
      }
      {
        float a0, b0, a1, b1;
        f2_unpack(rs2[0], a0, b0);
        f2_unpack(rs2[1], a1, b1);
        l += (a0 + b0) + (a1 + b1);
      }
      {   // P_j as packed bf16 pairs over the first 32 columns of its S buffer
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) pk[i] = pack_bf16(sv[2 * i], sv[2 * i + 1]);
        tmem_st32(tmem + lane_base + st * FBKV, pk);
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    if (ok && mbar_wait(o_final, 0)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool valid = qi < len;
      __nv_bfloat16* orow = p.o + ((size_t)(s0 + qi) * p.Hq + h) * D;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + T_O + c * 32, r);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint4 u;
            u.x = pack_bf16(__uint_as_float(r[8 * i + 0]) * inv, __uint_as_float(r[8 * i + 1]) * inv);
            u.y = pack_bf16(__uint_as_float(r[8 * i + 2]) * inv, __uint_as_float(r[8 * i + 3]) * inv);
            u.z = pack_bf16(__uint_as_float(r[8 * i + 4]) * inv, __uint_as_float(r[8 * i + 5]) * inv);
            u.w = pack_bf16(__uint_as_float(r[8 * i + 6]) * inv, __uint_as_float(r[8 * i + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * i) = u;
          }
        }
      }
      if (valid) p.lse[(size_t)h * p.T + s0 + qi] = (m + __log2f(l)) * 0.6931471805599453f;
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kFwdTmemCols);
  }
}


// ============================================================== backward
// delta[h, t] = sum_d dO[t,h,d] * O[t,h,d];  also zeroes the fp32 dQ accumulator.
__global__ void attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ dO, int ld_do,
                                     const __nv_bfloat16* __restrict__ O, int Hq, int T,
                                     float* __restrict__ delta, float* __restrict__ dq_acc) {
  const long gw = (long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (gw >= (long)T * Hq) return;
  const int t = gw / Hq, h = gw % Hq;
  const __nv_bfloat16* a = dO + (size_t)t * ld_do + h * D + lane * 4;
  const __nv_bfloat16* b = O + ((size_t)t * Hq + h) * D + lane * 4;
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) s += __bfloat162float(a[e]) * __bfloat162float(b[e]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  if (lane == 0) delta[(size_t)h * T + t] = s;
  *reinterpret_cast<float4*>(dq_acc + ((size_t)t * Hq + h) * D + lane * 4) = make_float4(0, 0, 0, 0);
}

__global__ void attn_dq_convert_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dq,
                                       int ld_dq, int Hq, int T) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // one thread per 8 elements
  const long total = (long)T * Hq * (D / 8);
  if (i >= total) return;
  const long row = i / (Hq * (D / 8));
  const int rem = i % (Hq * (D / 8));
  const float* src = dq_acc + row * (long)Hq * D + rem * 8;
  float4 a = *reinterpret_cast<const float4*>(src);
  float4 b = *reinterpret_cast<const float4*>(src + 4);
  uint4 u;
  u.x = pack_bf16(a.x, a.y);
  u.y = pack_bf16(a.z, a.w);
  u.z = pack_bf16(b.x, b.y);
  u.w = pack_bf16(b.z, b.w);
  *reinterpret_cast<uint4*>(dq + row * (long)ld_dq + rem * 8) = u;
}

struct BwdParams {
  const int* cu_seqlens;
  int nseq, nkblk;
  int Hq, Hkv;
  float scale, scale_log2;
  const float* lse;    // [Hq, T] natural log
  const float* delta;  // [Hq, T]
  float* dq_acc;       // [T, Hq, D] fp32, pre-zeroed
  __nv_bfloat16* dk;   // [T, Hkv, D] (row stride ld_dk)
  __nv_bfloat16* dv;
  int ld_dk, ld_dv;
  int T;
};

// Backward tiling: one CTA per (128-row key block, kv head); per iteration a
// 64-row query block of one query head of the GQA group.
constexpr int BQB = 64;                           // query rows per backward iteration
constexpr int QTILE_BYTES = BQB * D * 2;          // 16 KB: 64 rows as two 8 KB swizzle atoms
constexpr int PTILE_BYTES = BKV * BQB * 2;        // 16 KB: 128 kv rows x 64 q cols, one atom
constexpr int kBwdThreads = 448;                  // producer, MMA, 8 softmax (two per kv row), 4 dQ warps

struct BwdSmem {
  static constexpr int K_OFF = 0;                             // 32 KB
  static constexpr int V_OFF = TILE_BYTES;                    // 32 KB
  static constexpr int Q_OFF = 2 * TILE_BYTES;                // 2 stages x 16 KB
  static constexpr int DO_OFF = Q_OFF + 2 * QTILE_BYTES;      // 2 stages x 16 KB
  static constexpr int PT_OFF = DO_OFF + 2 * QTILE_BYTES;     // 2 buffers x 16 KB
  static constexpr int DS_OFF = PT_OFF + 2 * PTILE_BYTES;     // 2 buffers x 16 KB
  static constexpr int DQ_OFF = DS_OFF + 2 * PTILE_BYTES;     // [64 q][128 d] fp32 dQ staging, 32 KB
  static constexpr int VEC_OFF = DQ_OFF + BQB * D * 4;         // [2][lse2 64 | delta 64]
  static constexpr int BAR_OFF = VEC_OFF + 1024;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
};
static_assert(BwdSmem::TOTAL <= 227 * 1024, "backward shared memory");

KORE_DEV void named_bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

// Write 32 values (columns [32c, 32c+32) of a tile row) as bf16 into a K-major SW128 tile.
KORE_DEV void store_row32_sw128(uint8_t* tile, int row, int c, const float* v) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int chunk = c * 4 + k;  // 0..15
    uint4 u;
    u.x = pack_bf16(v[8 * k + 0], v[8 * k + 1]);
    u.y = pack_bf16(v[8 * k + 2], v[8 * k + 3]);
    u.z = pack_bf16(v[8 * k + 4], v[8 * k + 5]);
    u.w = pack_bf16(v[8 * k + 6], v[8 * k + 7]);
    uint8_t* atom = tile + (chunk >> 3) * 16384;
    *reinterpret_cast<uint4*>(atom + row * 128 + (((chunk & 7) ^ (row & 7)) * 16)) = u;
  }
}

// Work item of a CTA: heaviest key blocks (kb = 0) of every kv head first.
struct BwdItem {
  int seq, kb, kvh;
};
KORE_DEV BwdItem bwd_item(const BwdParams& p) {
  const int x = blockIdx.x;
  BwdItem it;
  it.kvh = x % p.Hkv;
  const int rest = x / p.Hkv;
  it.kb = rest / p.nseq;
  it.seq = rest % p.nseq;
  return it;
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, BwdParams p) {
  using S = BwdSmem;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;     // S^T, dP^T of this iteration in TMEM
  uint64_t* s_free = bars + 6;     // softmax warps have read them
  uint64_t* p_full = bars + 7;     // [2] P^T, dS^T in shared memory
  uint64_t* p_empty = bars + 9;    // [2] the gradient MMAs that read them completed
  uint64_t* dq_full = bars + 11;
  uint64_t* dq_empty = bars + 12;
  uint64_t* all_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_vec = reinterpret_cast<float*>(smem + S::VEC_OFF);  // [2][128]: lse2[64], delta[64]

  const BwdItem item = bwd_item(p);
  const int seq = item.seq, kb = item.kb, kvh = item.kvh;
  const int G = p.Hq / p.Hkv;
  const int s0 = p.cu_seqlens[seq];
  const int len = p.cu_seqlens[seq + 1] - s0;
  const int k0 = kb * BKV;
  if (k0 >= len) return;
  const int nqb = (len + BQB - 1) / BQB;
  const int qb0 = k0 / BQB;           // first causal query block (2 * kb)
  const int per_head = nqb - qb0;
  const int iters = G * per_head;
  const int warp = threadIdx.x / 32;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 4);
    mbar_init(all_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: [0,64) S^T, [64,128) dP^T, [128,192) dQ^T (lanes = head dim), [256,384) dV, [384,512) dK
  constexpr uint32_t T_S = 0, T_DP = 64, T_DQ = 128, T_DV = 256, T_DK = 384;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_2d(smem + S::K_OFF, &tmK, kv_full, kvh * D, s0 + k0);
      tma_load_2d(smem + S::K_OFF + 16384, &tmK, kv_full, kvh * D + 64, s0 + k0);
      tma_load_2d(smem + S::V_OFF, &tmV, kv_full, kvh * D, s0 + k0);
      tma_load_2d(smem + S::V_OFF + 16384, &tmV, kv_full, kvh * D + 64, s0 + k0);
      for (int i = 0; i < iters && !*abort_flag; ++i) {
        const int st = i & 1;
        const int h = kvh * G + i / per_head;
        const int q0 = (qb0 + i % per_head) * BQB;
        if (!mbar_wait(&qdo_empty[st], ((i >> 1) & 1) ^ 1)) { *abort_flag = 1; break; }
        mbar_arrive_expect_tx(&qdo_full[st], 2 * QTILE_BYTES);
        uint8_t* qs = smem + S::Q_OFF + st * QTILE_BYTES;
        uint8_t* ds = smem + S::DO_OFF + st * QTILE_BYTES;
        tma_load_2d(qs, &tmQ, &qdo_full[st], h * D, s0 + q0);
        tma_load_2d(qs + 8192, &tmQ, &qdo_full[st], h * D + 64, s0 + q0);
        tma_load_2d(ds, &tmDO, &qdo_full[st], h * D, s0 + q0);
        tma_load_2d(ds + 8192, &tmDO, &qdo_full[st], h * D + 64, s0 + q0);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    constexpr uint32_t id_s = make_idesc_bf16(128, BQB, false, false);   // K Q^T, V dO^T
    constexpr uint32_t id_dv = make_idesc_bf16(128, 128, false, true);   // P^T dO, dS^T Q
    constexpr uint32_t id_dq = make_idesc_bf16(128, BQB, true, true);    // K^T dS^T = dQ^T
    if (elect_one()) {
      const uint32_t ka = smem_u32(smem + S::K_OFF), va = smem_u32(smem + S::V_OFF);
      bool ok = mbar_wait(kv_full, 0);
      // gradient MMAs of iteration j (reads P^T/dS^T buffer j%2 and Q/dO stage j%2)
      auto grads = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&p_full[st], (j >> 1) & 1)) return false;
        if (j > 0 && !mbar_wait(dq_empty, (j - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + S::Q_OFF + st * QTILE_BYTES);
        const uint32_t da = smem_u32(smem + S::DO_OFF + st * QTILE_BYTES);
        const uint32_t pa = smem_u32(smem + S::PT_OFF + st * PTILE_BYTES);
        const uint32_t sa = smem_u32(smem + S::DS_OFF + st * PTILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BQB / 16; ++kk) {
          const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ss(tmem + T_DV, kmajor_narrow_desc(pa, kk), mnmajor64_desc(da, kk), id_dv, acc);
          umma_f16_ss(tmem + T_DK, kmajor_narrow_desc(sa, kk), mnmajor64_desc(qa, kk), id_dv, acc);
        }
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_f16_ss(tmem + T_DQ, mnmajor_desc(ka, kk), mnmajor_narrow_desc(sa, kk), id_dq, kk > 0);
        umma_commit(&qdo_empty[st]);
        umma_commit(&p_empty[st]);
        umma_commit(dq_full);
        return true;
      };
      for (int i = 0; i < iters && ok; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&qdo_full[st], (i >> 1) & 1)) { ok = false; break; }
        if (i > 0 && !mbar_wait(s_free, (i - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + S::Q_OFF + st * QTILE_BYTES);
        const uint32_t da = smem_u32(smem + S::DO_OFF + st * QTILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          umma_f16_ss(tmem + T_S, kmajor_desc(ka, kk), kmajor64_desc(qa, kk), id_s, kk > 0);
          umma_f16_ss(tmem + T_DP, kmajor_desc(va, kk), kmajor64_desc(da, kk), id_s, kk > 0);
        }
        umma_commit(s_full);
        if (i > 0 && !grads(i - 1)) { ok = false; break; }
      }
      if (ok && iters > 0 && !grads(iters - 1)) ok = false;
      if (ok) umma_commit(all_done);
      else *abort_flag = 1;
    }
    __syncwarp();
  } else if (warp < 10) {
    // ---- softmax warps: two per kv row, each on 32 of the 64 query columns
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;
    const int lane = threadIdx.x & 31;
    const int row = q4 * 32 + lane;
    const int tid = threadIdx.x - 64;  // 0..255; 0..127 also stage lse2 / delta
    const int kvi = k0 + row;
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    bool ok = true;
    auto vec_load = [&](int i) -> float {  // lse2 (tid < 64) or delta (64 <= tid < 128) of iteration i
      if (tid >= 128) return 0.f;
      const int h = kvh * G + i / per_head;
      const int qi = (qb0 + i % per_head) * BQB + (tid & 63);
      if (qi >= len) return tid < 64 ? INFINITY : 0.f;
      return tid < 64 ? p.lse[(size_t)h * p.T + s0 + qi] * kLog2e : p.delta[(size_t)h * p.T + s0 + qi];
    };
    if (iters > 0 && tid < 128) s_vec[tid] = vec_load(0);
    // after a failed wait the loop keeps running (no waits, no work) so every
    // softmax thread still reaches each named barrier
    for (int i = 0; i < iters; ++i) {
      const int q0 = (qb0 + i % per_head) * BQB;
      const int st = i & 1;
      const float nxt = (i + 1 < iters) ? vec_load(i + 1) : 0.f;   // prefetch next iteration's statistics
      named_bar_sync(1, 256);
      if (!ok) continue;
      const float* lse2 = s_vec + st * 128 + half * 32;
      const float* dlt = s_vec + st * 128 + 64 + half * 32;
      if (!mbar_wait(s_full, i & 1)) { ok = false; *abort_flag = 1; continue; }
      tc_fence_after();
      uint32_t rs[32], rp[32];
      tmem_ld32(tmem + lane_base + T_S + half * 32, rs);
      tmem_ld32(tmem + lane_base + T_DP + half * 32, rp);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      if (!mbar_wait(&p_empty[st], ((i >> 1) & 1) ^ 1)) { ok = false; *abort_flag = 1; continue; }
      const bool diag = q0 < k0 + BKV;
      // P and dS overwrite the raw registers in place (no extra live arrays)
      float* pv = reinterpret_cast<float*>(rs);
      float* dv = reinterpret_cast<float*>(rp);
      // P^T = 2^(S^T scale_log2 - lse2), dS^T = P^T (dP^T - delta): packed pairs
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2);
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const int qc = half * 32 + e;
        float a0, a1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(rs[e]), __uint_as_float(rs[e + 1])), sc2,
                         f2_pack(-lse2[e], -lse2[e + 1])), a0, a1);
        float pr0 = exp2f(a0), pr1 = exp2f(a1);
        if ((diag && q0 + qc < kvi) || kvi >= len) pr0 = 0.f;
        if ((diag && q0 + qc + 1 < kvi) || kvi >= len) pr1 = 0.f;
        const uint64_t pp = f2_pack(pr0, pr1);
        f2_unpack(f2_mul(pp, f2_add(f2_pack(__uint_as_float(rp[e]), __uint_as_float(rp[e + 1])),
                                    f2_pack(-dlt[e], -dlt[e + 1]))), dv[e], dv[e + 1]);
        pv[e] = pr0;
        pv[e + 1] = pr1;
      }
      store_row32_sw128(smem + S::PT_OFF + st * PTILE_BYTES, row, half, pv);
      store_row32_sw128(smem + S::DS_OFF + st * PTILE_BYTES, row, half, dv);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
      if (tid < 128) s_vec[(st ^ 1) * 128 + tid] = nxt;   // buffer st^1 was last read in iteration i-1
    }
    if (ok && iters > 0 && mbar_wait(all_done, 0)) {
      tc_fence_after();
      const bool valid = kvi < len;
      __nv_bfloat16* dvrow = p.dv + (size_t)(s0 + kvi) * p.ld_dv + kvh * D;
      __nv_bfloat16* dkrow = p.dk + (size_t)(s0 + kvi) * p.ld_dk + kvh * D;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        __nv_bfloat16* out = part == 0 ? dvrow : dkrow;
        const float mul = part == 0 ? 1.f : p.scale;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c = half * 2 + cc;   // this warp's 64 of the 128 head-dim columns
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + (part == 0 ? T_DV : T_DK) + c * 32, r);
          tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint4 u;
              u.x = pack_bf16(__uint_as_float(r[8 * k + 0]) * mul, __uint_as_float(r[8 * k + 1]) * mul);
              u.y = pack_bf16(__uint_as_float(r[8 * k + 2]) * mul, __uint_as_float(r[8 * k + 3]) * mul);
              u.z = pack_bf16(__uint_as_float(r[8 * k + 4]) * mul, __uint_as_float(r[8 * k + 5]) * mul);
              u.w = pack_bf16(__uint_as_float(r[8 * k + 6]) * mul, __uint_as_float(r[8 * k + 7]) * mul);
              *reinterpret_cast<uint4*>(out + c * 32 + 8 * k) = u;
            }
          }
        }
      }
    } else if (iters > 0) {
      *abort_flag = 1;
    }
  } else {
    // ---- dQ warps: one head-dim lane per thread; dQ^T columns are query rows.
    // The 64 x 128 fp32 partial goes through shared memory into one TMA
    // reduce-add per iteration (whole 512-byte rows, no per-element atomics).
    const int q4 = warp & 3;
    const int lane = threadIdx.x & 31;
    const int d = q4 * 32 + lane;
    const bool leader = threadIdx.x == 10 * 32;
    float* stage = reinterpret_cast<float*>(smem + S::DQ_OFF);
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    bool ok = true;
    for (int j = 0; j < iters; ++j) {
      const int h = kvh * G + j / per_head;
      const int q0 = (qb0 + j % per_head) * BQB;
      uint32_t r[2][32];
      if (ok && !mbar_wait(dq_full, j & 1)) { ok = false; *abort_flag = 1; }
      if (ok) {
        tc_fence_after();
        tmem_ld32(tmem + lane_base + T_DQ, r[0]);
        tmem_ld32(tmem + lane_base + T_DQ + 32, r[1]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
      }
      if (leader) tma_store_wait_read<0>();   // the previous reduce has read the staging buffer
      named_bar_sync(2, 128);
      if (ok) {
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) stage[(c * 32 + e) * D + d] = __uint_as_float(r[c][e]) * p.scale;
      }
      fence_proxy_async_smem();
      named_bar_sync(2, 128);
      // rows past the sequence hold exact zeros (their dS is zero), so adding
      // them into the next sequence's rows changes nothing; rows past T are clipped
      if (ok && leader) {
        tma_reduce_add_3d(&tmDQ, stage, 0, h, s0 + q0);
        tma_store_commit();
      }
    }
    if (leader) tma_store_wait_all<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Host launch shared by the allocating and the allocation-free entry points.
// tmQ / tmDO: 64-row boxes; tmK / tmV: 128-row boxes.
inline cudaError_t launch_bwd_main(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                                   const CUtensorMap& tdo, const BwdParams& p, cudaStream_t st) {
  // dQ accumulator [T, Hq, 128] fp32 as a 3-D map (d, head, token) for the reduce-add boxes
  CUtensorMap tdq;
  try {
    tdq = make_tmap_3d(p.dq_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, p.Hq, p.T, D, (uint64_t)p.Hq * D, D, 1, BQB,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  } catch (...) {   // callers include a C entry point: no exceptions across it
    return cudaErrorInvalidValue;
  }
  static bool attr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {   // the attribute is per device
    e = cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BwdSmem::TOTAL);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  attn_bwd_kernel<<<p.nseq * p.nkblk * p.Hkv, kBwdThreads, BwdSmem::TOTAL, st>>>(tq, tk, tv, tdo, tdq, p);
  return cudaGetLastError();
}

void check_qkv(const at::Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 3 && t.size(2) == D &&
                  t.stride(2) == 1 && t.stride(1) == D,
              n, ": expected bf16 [T, H, 128] with contiguous heads");
  TORCH_CHECK(t.stride(0) % 8 == 0, n, ": row stride must be a multiple of 8 elements");
}

}  // namespace attn

void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
              const at::Tensor& cu_seqlens, int64_t max_seqlen, double scale, at::Tensor& o,
              at::Tensor& lse) {
  using namespace attn;
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  TORCH_CHECK(o.is_contiguous() && o.scalar_type() == at::kBFloat16, "o must be contiguous bf16");
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat, "lse must be fp32");
  TORCH_CHECK(cu_seqlens.scalar_type() == at::kInt && cu_seqlens.is_cuda(), "cu_seqlens int32 cuda");
  const int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  TORCH_CHECK(Hq % Hkv == 0, "GQA: Hq must be a multiple of Hkv");
  const int nseq = cu_seqlens.numel() - 1;
  if (T == 0 || nseq <= 0) return;
  c10::cuda::CUDAGuard g(q.device());
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq = make_tmap_2d(q.data_ptr(), bf, 2, (uint64_t)Hq * D, T, q.stride(0), 64, 128);
  CUtensorMap tk = make_tmap_2d(k.data_ptr(), bf, 2, (uint64_t)Hkv * D, T, k.stride(0), 64, FBKV);
  CUtensorMap tv = make_tmap_2d(v.data_ptr(), bf, 2, (uint64_t)Hkv * D, T, v.stride(0), 64, FBKV);
  FwdParams p;
  p.cu_seqlens = cu_seqlens.data_ptr<int>();
  p.nseq = nseq;
  p.nqblk = (int)((max_seqlen + BQ - 1) / BQ);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = (float)scale * kLog2e;
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.T = T;
  constexpr int smem = FwdSmem::TOTAL;
  static bool attr[64] = {};
  const int dev = q.get_device();
  TORCH_CHECK(dev >= 0 && dev < 64, "attn_fwd: device index");
  if (!attr[dev]) {
    check_cuda(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "attn_fwd smem attr");
    // two CTAs per SM: ask for the full shared-memory carveout
    check_cuda(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100),
               "attn_fwd carveout");
    attr[dev] = true;
  }
  dim3 grid(nseq * p.nqblk, Hq);
  attn_fwd_kernel<<<grid, kThreads, smem, at::cuda::getCurrentCUDAStream()>>>(tq, tk, tv, p);
  check_cuda(cudaGetLastError(), "attn_fwd launch");
}

// dq/dk/dv may be strided views [T, H, 128] of larger buffers.
// dq_acc: fp32 scratch [T, Hq, 128] (zeroed here), delta: fp32 scratch [Hq, T].
void attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
              const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
              const at::Tensor& cu_seqlens, int64_t max_seqlen, double scale, at::Tensor& dq,
              at::Tensor& dk, at::Tensor& dv, at::Tensor& dq_acc, at::Tensor& delta) {
  using namespace attn;
  check_qkv(dout, "dout");
  check_qkv(q, "q");
  check_qkv(k, "k");
  check_qkv(v, "v");
  check_qkv(dq, "dq");
  check_qkv(dk, "dk");
  check_qkv(dv, "dv");
  TORCH_CHECK(o.is_contiguous(), "o must be contiguous [T, Hq, 128]");
  const int T = q.size(0), Hq = q.size(1), Hkv = k.size(1);
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.numel() >= (int64_t)T * Hq * D,
              "dq_acc must be fp32 with T*Hq*128 elements");
  TORCH_CHECK(delta.scalar_type() == at::kFloat && delta.numel() >= (int64_t)T * Hq,
              "delta must be fp32 with Hq*T elements");
  const int nseq = cu_seqlens.numel() - 1;
  if (T == 0 || nseq <= 0) return;
  c10::cuda::CUDAGuard g(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  {
    const long warps = (long)T * Hq;
    attn_bwd_prep_kernel<<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), Hq, T, delta.data_ptr<float>(),
        dq_acc.data_ptr<float>());
    check_cuda(cudaGetLastError(), "attn_bwd_prep");
  }
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap tq = make_tmap_2d(q.data_ptr(), bf, 2, (uint64_t)Hq * D, T, q.stride(0), 64, BQB);
  CUtensorMap tk = make_tmap_2d(k.data_ptr(), bf, 2, (uint64_t)Hkv * D, T, k.stride(0), 64, 128);
  CUtensorMap tv = make_tmap_2d(v.data_ptr(), bf, 2, (uint64_t)Hkv * D, T, v.stride(0), 64, 128);
  CUtensorMap tdo = make_tmap_2d(dout.data_ptr(), bf, 2, (uint64_t)Hq * D, T, dout.stride(0), 64, BQB);
  BwdParams p;
  p.cu_seqlens = cu_seqlens.data_ptr<int>();
  p.nseq = nseq;
  p.nkblk = (int)((max_seqlen + BKV - 1) / BKV);
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = (float)scale;
  p.scale_log2 = (float)scale * kLog2e;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.ld_dk = dk.stride(0);
  p.ld_dv = dv.stride(0);
  p.T = T;
  check_cuda(launch_bwd_main(tq, tk, tv, tdo, p, st), "attn_bwd launch");
  const long n8 = (long)T * Hq * (D / 8);
  attn_dq_convert_kernel<<<(int)((n8 + 255) / 256), 256, 0, st>>>(
      dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), dq.stride(0), Hq, T);
  check_cuda(cudaGetLastError(), "attn_dq_convert");
}

}  // namespace kore

// ============================================================== allocation-free variant
// See attention_noalloc.h: same kernels as kore::attn_bwd, with the scratch
// (fp32 dQ accumulator + delta) in a fixed device array instead of
// caller-provided tensors. Nothing here allocates memory.
#include <mutex>

#include "attention_noalloc.h"

namespace kore {
namespace attn {

static __device__ __align__(256) unsigned char g_noalloc_scratch[KORE_ATTN_NOALLOC_SCRATCH_BYTES];

struct NoallocDeviceState {
  void* scratch = nullptr;  // device address of g_noalloc_scratch on this device
};

static int noalloc_setup(int dev, NoallocDeviceState** out) {
  static std::mutex mu;
  static NoallocDeviceState states[64];
  if (dev < 0 || dev >= 64) return KORE_NOALLOC_ERR_SETUP;
  std::lock_guard<std::mutex> lock(mu);
  NoallocDeviceState& s = states[dev];
  if (s.scratch == nullptr) {
    // host code must not use the array's name as an address: ask the runtime
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
      return KORE_NOALLOC_ERR_SETUP;
    s.scratch = ptr;
  }
  *out = &s;
  return KORE_NOALLOC_OK;
}

}  // namespace attn
}  // namespace kore

extern "C" int kore_attn_bwd_noalloc(const void* dout, int64_t ld_dout, const void* q,
                                     int64_t ld_q, const void* k, int64_t ld_k, const void* v,
                                     int64_t ld_v, const void* o, const float* lse,
                                     const int* cu_seqlens, int nseq, int max_seqlen, int T,
                                     int Hq, int Hkv, float scale, void* dq, int64_t ld_dq,
                                     void* dk, int64_t ld_dk, void* dv, int64_t ld_dv,
                                     cudaStream_t stream) {
  using namespace kore;
  using namespace kore::attn;
  if (T <= 0 || nseq <= 0 || max_seqlen <= 0 || max_seqlen > T || Hq <= 0 || Hkv <= 0 || Hq % Hkv != 0)
    return KORE_NOALLOC_ERR_ARGS;
  // row strides: multiples of 8 elements, at least one row wide, and within int range
  const int64_t wq = (int64_t)Hq * D, wk = (int64_t)Hkv * D;
  const int64_t ld[7] = {ld_dout, ld_q, ld_dq, ld_k, ld_v, ld_dk, ld_dv};
  const int64_t width[7] = {wq, wq, wq, wk, wk, wk, wk};
  for (int i = 0; i < 7; ++i)
    if (ld[i] % 8 != 0 || ld[i] < width[i] || ld[i] > INT32_MAX) return KORE_NOALLOC_ERR_ARGS;
  // tensors read by TMA or 16-byte vectors need 16-byte alignment; lse and
  // cu_seqlens are read element-wise and need 4
  const void* ptrs16[8] = {dout, q, k, v, o, dq, dk, dv};
  for (const void* ptr : ptrs16)
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return KORE_NOALLOC_ERR_ARGS;
  const void* ptrs4[2] = {lse, cu_seqlens};
  for (const void* ptr : ptrs4)
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 3) != 0) return KORE_NOALLOC_ERR_ARGS;
  // the backward grid is nseq * ceil(max_seqlen / 128) * Hkv CTAs
  if ((int64_t)nseq * ((max_seqlen + BKV - 1) / BKV) * Hkv > INT32_MAX) return KORE_NOALLOC_ERR_ARGS;
  const uint64_t acc_bytes = (uint64_t)T * Hq * D * sizeof(float);
  const uint64_t delta_bytes = (uint64_t)T * Hq * sizeof(float);
  if (acc_bytes + delta_bytes > KORE_ATTN_NOALLOC_SCRATCH_BYTES) return KORE_NOALLOC_ERR_TOO_LARGE;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return KORE_NOALLOC_ERR_SETUP;
  NoallocDeviceState* st = nullptr;
  int rc = noalloc_setup(dev, &st);
  if (rc != KORE_NOALLOC_OK) return rc;
  float* dq_acc = reinterpret_cast<float*>(st->scratch);
  float* delta = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(st->scratch) + acc_bytes);
  CUtensorMap tq, tk, tv, tdo;
  try {
    auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    tq = make_tmap_2d(q, bf, 2, (uint64_t)Hq * D, T, ld_q, 64, BQB);
    tk = make_tmap_2d(k, bf, 2, (uint64_t)Hkv * D, T, ld_k, 64, 128);
    tv = make_tmap_2d(v, bf, 2, (uint64_t)Hkv * D, T, ld_v, 64, 128);
    tdo = make_tmap_2d(dout, bf, 2, (uint64_t)Hq * D, T, ld_dout, 64, BQB);
  } catch (...) {
    return KORE_NOALLOC_ERR_ARGS;
  }
  // delta and a zeroed dQ accumulator (the array keeps the previous call's data)
  {
    const long warps = (long)T * Hq;
    attn_bwd_prep_kernel<<<(int)((warps * 32 + 255) / 256), 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout), (int)ld_dout,
        reinterpret_cast<const __nv_bfloat16*>(o), Hq, T, delta, dq_acc);
    if (cudaGetLastError() != cudaSuccess) return KORE_NOALLOC_ERR_LAUNCH;
  }
  BwdParams p;
  p.cu_seqlens = cu_seqlens;
  p.nseq = nseq;
  p.nkblk = (max_seqlen + BKV - 1) / BKV;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.ld_dk = (int)ld_dk;
  p.ld_dv = (int)ld_dv;
  p.T = T;
  if (launch_bwd_main(tq, tk, tv, tdo, p, stream) != cudaSuccess) return KORE_NOALLOC_ERR_LAUNCH;
  const long n8 = (long)T * Hq * (D / 8);
  attn_dq_convert_kernel<<<(int)((n8 + 255) / 256), 256, 0, stream>>>(
      dq_acc, reinterpret_cast<__nv_bfloat16*>(dq), (int)ld_dq, Hq, T);
  if (cudaGetLastError() != cudaSuccess) return KORE_NOALLOC_ERR_LAUNCH;
  return KORE_NOALLOC_OK;
}

// Reads and clears the device-side error word of the attention kernels (0 =
// no error, 1 = a bounded wait inside a kernel timed out and its outputs are
// incomplete). Synchronizes the current device.
extern "C" int kore_attn_noalloc_read_error(void) {
  int v = 0, z = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, kore::g_error, sizeof(int)) != cudaSuccess) return -1;
  if (cudaMemcpyToSymbol(kore::g_error, &z, sizeof(int)) != cudaSuccess) return -1;
  return v;
}
