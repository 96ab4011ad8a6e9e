// Persistent warp-specialized bf16 GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
//   C[M,N] (=|+=) alpha * op(A)[M,K] . op(B)[N,K]^T  (+ R[M,N])
//
// A is either K-major ([M,K] row-major) or MN-major ([K,M] row-major); the same
// for B ([N,K] or [K,N]). The three combinations cover a linear layer's
// forward (y = x W^T), data gradient (dx = dy W) and weight gradient
// (dW = dy^T x) without any transpose copies: UMMA reads MN-major operands
// straight from the 128B-swizzled tiles TMA writes.
//
// CTA layout (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one elected lane)
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  epilogue: tcgen05.ld -> fp32 math -> bf16/fp32 -> smem -> TMA store
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1. Every wait is bounded.
//
// Reference parity: the reference runs every linear layer through
// nn.Linear/cuBLAS inside HF transformers (kore/policy/sft.py:288-293,
// kore/policy/grpo.py:2017-2018); this kernel is the replacement hot path.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "tma_host.h"

namespace kore {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
// expert-parallel pull dispatch: four more warps per CTA stage the receive
// rows while the producer, MMA and epilogue warps run the GEMM
constexpr int kCopyWarps = 4;
constexpr int kThreadsPull = kThreads + 32 * kCopyWarps;
constexpr int kStageBytesC = 32 * 128;  // one epilogue staging buffer: 32 rows x 128 B

struct Params {
  int M, N, K;
  float alpha;
  int accumulate;       // C += result (reads old C)
  int out_f32;          // C is fp32 (else bf16)
  const void* C_read;   // C base pointer for accumulate reads
  int ldc;              // C row stride (elements)
  const __nv_bfloat16* R;  // optional residual (bf16, row stride ldr)
  int ldr;
  // grouped mode (MoE experts): per M-tile {expert, first row, row limit, 0};
  // B is a 3-D tensor map indexed by expert; rows >= limit are not stored.
  const int4* tiles;
  void* C_write;  // output base for the masked direct-store epilogue (grouped mode)
  // tensor-parallel all-gather->GEMM: A rows [i*ag_rows, (i+1)*ag_rows) live on
  // peer i (ag_src[i], row stride ag_lda). At kernel start every CTA copies
  // its share of 64-row groups into the local staging buffer ag_stage [M, K]
  // (each remote row crosses NVLink once) and publishes ag_flags[g] = ag_epoch;
  // a tile's producer waits for its groups, then TMA-loads A from ag_stage.
  int ag_rows;
  const void* ag_src[8] = {};
  void* ag_stage = nullptr;
  int* ag_flags = nullptr;
  int ag_epoch = 0;
  int ag_lda = 0;
  int ag_rot = 0;   // M-block rotation so each rank starts on its own (local) rows
  // expert-parallel pull dispatch (grouped mode): staged row r is a copy of row
  // (ag_index[r] & 0x3FFFFFF) of peer (ag_index[r] >> 26)'s token buffer
  // ag_src[peer] (row stride ag_lda), or zeros for ag_index[r] < 0 (pad rows);
  // only rows [0, min(*ag_rows_dev, ag_cap)) are staged (64-row groups)
  const int* ag_index = nullptr;
  const int* ag_rows_dev = nullptr;
  int ag_cap = 0;
  // tensor-parallel GEMM->reduce-scatter: output row r is stored (P2P) into
  // peer r / rs_rows, slot rs_rank, i.e. rs_out[peer] + (rs_rank*rs_rows + r%rs_rows)*ldc.
  int rs_rows;
  int rs_rank;
  void* rs_out[8];
  // split-K (skinny problems such as decode, M <= a few hundred rows): work unit
  // t covers output tile t % (num_m*num_n) over K blocks of split t / (num_m*num_n);
  // the fp32 partial tile goes to rows split*ws_rows + m of the workspace map tmC
  int splits = 1;
  int ws_rows = 0;
  // grouped mode with a device-built tile table: the number of M tiles is read
  // from device memory (no host round trip); p.M is the table's capacity
  const int* ntiles_dev = nullptr;
  // grouped weight-gradient mode (MoE experts): work item t covers expert
  // t / (num_m*num_n); its K range is rows [wg_offs[e], wg_offs[e+1]) of the
  // expert-major operands (multiples of 64); output rows are e * M + row
  const int* wg_offs = nullptr;
  int wg_E = 0;
};

// K blocks [kb0, kb1) of split s when `kblocks` are divided over `splits`.
KORE_DEV void split_range(int s, int splits, int kblocks, int& kb0, int& kb1) {
  kb0 = (int)(((long)s * kblocks) / splits);
  kb1 = (int)(((long)(s + 1) * kblocks) / splits);
}

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + kEpiWarps * 2 * kStageBytesC;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;  // + barriers + alignment slack
};

KORE_DEV void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  constexpr int G = 8;
  int per_group = G * num_n;
  int g = t / per_group;
  int first_m = g * G;
  int gsize = min(num_m - first_m, G);
  int r = t - g * per_group;
  tm = first_m + r % gsize;
  tn = r / gsize;
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreadsPull, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, Params p) {
  using S = Smem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int num_m = p.ntiles_dev != nullptr ? min(*p.ntiles_dev, (p.M + BM - 1) / BM) : (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_mn = num_m * num_n;
  const int num_tiles = p.wg_offs != nullptr ? num_mn * p.wg_E : num_mn * p.splits;
  const int kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // rows of A that the staging copy fills (flag waits never look past them)
  const int stage_rows = p.ag_index != nullptr ? min(min(*p.ag_rows_dev, p.ag_cap), p.M) : p.M;
  if (p.ag_flags != nullptr && p.ag_index == nullptr) {
    // ---------------------------------------------- staged all-gather copy
    // 64-row groups round-robin over CTAs; 8 outstanding 16-byte loads per
    // thread keep enough peer reads in flight to fill the NVLink pipe.
    const int groups = p.M / 64;
    const int vpr = p.K / 8;                 // 16-byte vectors per row
    const int total = 64 * vpr;
    for (int g = blockIdx.x; g < groups; g += gridDim.x) {
      const int owner = (g * 64) / p.ag_rows;
      const int lr = g * 64 - owner * p.ag_rows;
      const uint4* src = reinterpret_cast<const uint4*>(
          reinterpret_cast<const __nv_bfloat16*>(p.ag_src[owner]) + (size_t)lr * p.ag_lda);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.ag_stage) + (size_t)g * 64 * p.K);
      const int sstride = p.ag_lda / 8;
      for (int base = threadIdx.x; base < total; base += kThreads * 8) {
        uint4 buf[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int idx = base + u * kThreads;
          if (idx < total) buf[u] = src[(size_t)(idx / vpr) * sstride + idx % vpr];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int idx = base + u * kThreads;
          if (idx < total) dst[(size_t)(idx / vpr) * vpr + idx % vpr] = buf[u];
        }
      }
      fence_proxy_async_global();
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        st_release_gpu_s32(&p.ag_flags[g], p.ag_epoch);
      }
    }
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int tm, tn, kb0, kb1;
        tile_coords(t % num_mn, num_m, num_n, tm, tn);
        if (p.wg_offs != nullptr) {
          kb0 = p.wg_offs[t / num_mn] / BK;
          kb1 = p.wg_offs[t / num_mn + 1] / BK;
          if (kb0 >= kb1) continue;          // expert without rows: no loads, no MMA, no store
        } else {
          split_range(t / num_mn, p.splits, kblocks, kb0, kb1);
        }
        if (p.ag_rot) tm = (tm + p.ag_rot) % num_m;
        int m0 = tm * BM, ex = 0;
        const int n0 = tn * BN;
        if (p.tiles != nullptr) {
          const int4 ti = p.tiles[tm];
          ex = ti.x;
          m0 = ti.y;
        }
        if (p.ag_flags != nullptr) {   // staged all-gather: this tile's row groups must be in ag_stage
          bool ready = true;
          for (int g = m0 / 64; g < min(m0 + BM, stage_rows) / 64 && ready; ++g)
            ready = wait_flag_ge(&p.ag_flags[g], p.ag_epoch);
          if (!ready) { *abort_flag = 1; break; }
          fence_proxy_async_global();    // generic-proxy copies -> TMA reads
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sA = smem + stage * S::STAGE_BYTES;
          uint8_t* sB = sA + S::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], S::STAGE_BYTES);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d(sA, &tmA, &full_bar[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(sA + j * 8192, &tmA, &full_bar[stage], m0 + 64 * j, k0);
          }
          if (p.tiles != nullptr) {  // per-expert weights: 3-D map (inner, outer, expert)
            if (!B_MN) {
              tma_load_3d(sB, &tmB, &full_bar[stage], k0, n0, ex);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_3d(sB + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0, ex);
            }
          } else if (!B_MN) {
            tma_load_2d(sB, &tmB, &full_bar[stage], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + j * 8192, &tmB, &full_bar[stage], n0 + 64 * j, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int kb0, kb1;
        if (p.wg_offs != nullptr) {
          kb0 = p.wg_offs[t / num_mn] / BK;
          kb1 = p.wg_offs[t / num_mn + 1] / BK;
          if (kb0 >= kb1) continue;
        } else {
          split_range(t / num_mn, p.splits, kblocks, kb0, kb1);
        }
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        ++it;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::STAGE_BYTES);
          const uint32_t b_addr = a_addr + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad = A_MN ? make_sw128_desc(a_addr + k * 2048, 8192, 1024)
                               : make_sw128_desc(a_addr + k * 32, 16, 1024);
            uint64_t bd = B_MN ? make_sw128_desc(b_addr + k * 2048, 8192, 1024)
                               : make_sw128_desc(b_addr + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb != kb0) || (k != 0));
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        umma_commit(&tfull_bar[acc]);
      }
    }
    __syncwarp();
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int lane = threadIdx.x & 31;
    uint8_t* stage_buf = smem + S::EPI_OFF + (warp - 2) * 2 * kStageBytesC;
    int buf = 0;
    int it = 0;
    const int CH = p.out_f32 ? 32 : 64;  // output columns per 128-byte staging row
    for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
      int tm, tn;
      tile_coords(t % num_mn, num_m, num_n, tm, tn);
      int ws_row0 = (t / num_mn) * p.ws_rows;   // split-K: this split's workspace rows
      if (p.wg_offs != nullptr) {
        const int e = t / num_mn;
        if (p.wg_offs[e] >= p.wg_offs[e + 1]) continue;
        ws_row0 = e * p.M;                      // expert e's block of the [E * M, N] gradient
      }
      if (p.ag_rot) tm = (tm + p.ag_rot) % num_m;
      int m0 = tm * BM, m_lim = p.M;
      const int n0 = tn * BN;
      if (p.tiles != nullptr) {
        const int4 ti = p.tiles[tm];
        m0 = ti.y;
        m_lim = ti.z;
      }
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      ++it;
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      for (int c0 = 0; c0 < BN; c0 += CH) {
        if (n0 + c0 >= p.N) break;
        float v[64];
        {
          uint32_t r[32];
          tmem_ld32(t_row + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
          if (!p.out_f32) {
            tmem_ld32(t_row + c0 + 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(r[i]) * p.alpha;
          }
        }
        const bool row_ok = row < m_lim;
        // optional accumulate / residual (row-contiguous per thread)
        if (row_ok && (p.accumulate || p.R != nullptr)) {
          const int ncols = min(CH, p.N - (n0 + c0));
          if (p.R != nullptr) {
            const __nv_bfloat16* rp = p.R + (size_t)row * p.ldr + n0 + c0;
#pragma unroll
            for (int j = 0; j < 64; j += 8) {
              if (j >= ncols) break;
              uint4 u = *reinterpret_cast<const uint4*>(rp + j);
              const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[j + e] += __bfloat162float(h[e]);
            }
          }
          if (p.accumulate) {
            if (p.out_f32) {
              const float* cp = reinterpret_cast<const float*>(p.C_read) + (size_t)(row + (p.wg_offs ? ws_row0 : 0)) * p.ldc + n0 + c0;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                if (j >= ncols) break;
                float4 u = *reinterpret_cast<const float4*>(cp + j);
                v[j] += u.x; v[j + 1] += u.y; v[j + 2] += u.z; v[j + 3] += u.w;
              }
            } else {
              const __nv_bfloat16* cp =
                  reinterpret_cast<const __nv_bfloat16*>(p.C_read) + (size_t)(row + (p.wg_offs ? ws_row0 : 0)) * p.ldc + n0 + c0;
#pragma unroll
              for (int j = 0; j < 64; j += 8) {
                if (j >= ncols) break;
                uint4 u = *reinterpret_cast<const uint4*>(cp + j);
                const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[j + e] += __bfloat162float(h[e]);
              }
            }
          }
        }
        if (p.tiles != nullptr || p.rs_rows > 0) {
          // grouped: masked direct stores (a tile may end inside another expert's rows);
          // reduce-scatter: the row goes to its owner peer's slot (P2P store)
          const int ncols = min(CH, p.N - (n0 + c0));
          size_t orow = (size_t)row;
          void* obase = p.C_write;
          if (p.rs_rows > 0) {
            obase = p.rs_out[row / p.rs_rows];
            orow = (size_t)p.rs_rank * p.rs_rows + row % p.rs_rows;
          }
          if (row_ok) {
            if (p.out_f32) {
              float* cp = reinterpret_cast<float*>(obase) + orow * p.ldc + n0 + c0;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                if (j >= ncols) break;
                *reinterpret_cast<float4*>(cp + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              }
            } else {
              __nv_bfloat16* cp = reinterpret_cast<__nv_bfloat16*>(obase) + orow * p.ldc + n0 + c0;
#pragma unroll
              for (int j = 0; j < 64; j += 8) {
                if (j >= ncols) break;
                *reinterpret_cast<uint4*>(cp + j) =
                    make_uint4(pack_bf16(v[j], v[j + 1]), pack_bf16(v[j + 2], v[j + 3]),
                               pack_bf16(v[j + 4], v[j + 5]), pack_bf16(v[j + 6], v[j + 7]));
              }
            }
          }
          continue;
        }
        // make sure the TMA store that last used this staging buffer has read it
        if (lane == 0) tma_store_wait_read<1>();
        __syncwarp();
        uint8_t* sb = stage_buf + buf * kStageBytesC + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 u;
          if (p.out_f32) {
            u.x = __float_as_uint(v[4 * j]);
            u.y = __float_as_uint(v[4 * j + 1]);
            u.z = __float_as_uint(v[4 * j + 2]);
            u.w = __float_as_uint(v[4 * j + 3]);
          } else {
            u.x = pack_bf16(v[8 * j], v[8 * j + 1]);
            u.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
          }
          *reinterpret_cast<uint4*>(sb + ((j ^ (lane & 7)) * 16)) = u;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, stage_buf + buf * kStageBytesC, n0 + c0, ws_row0 + m0 + q * 32);
          tma_store_commit();
        }
        buf ^= 1;
      }
      // accumulator fully read: hand it back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  } else if (p.ag_index != nullptr) {
    // ------------------------------------- expert-parallel pull dispatch copy
    // (copy warps, launched only in this mode) 64-row groups round-robin over
    // CTAs, in the order the tiles consume them; each row comes from the peer
    // and token row its index entry names (pad rows are zero-filled). The
    // group's 64 entries are read once into shared memory; 16 outstanding
    // 16-byte loads per thread keep NVLink reads in flight. A group's flag is
    // released after its rows are written; tiles wait for their groups.
    __shared__ int s_codes[64];
    const int ct = threadIdx.x - 32 * (2 + kEpiWarps);     // 0 .. 32 * kCopyWarps - 1
    constexpr int CT = 32 * kCopyWarps;
    const int groups = stage_rows / 64;
    const int vpr = p.K / 8;
    const int total = 64 * vpr;
    const int sstride = p.ag_lda / 8;
    for (int g = blockIdx.x; g < groups; g += gridDim.x) {
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.ag_stage) + (size_t)g * 64 * p.K);
      asm volatile("bar.sync 1, %0;" ::"r"(CT));           // the previous group's entries are no longer read
      if (ct < 64) s_codes[ct] = p.ag_index[g * 64 + ct];
      asm volatile("bar.sync 1, %0;" ::"r"(CT));
      for (int base = ct; base < total; base += CT * 16) {
        uint4 buf[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int idx = base + u * CT;
          if (idx < total) {
            const int code = s_codes[idx / vpr];
            if (code < 0) {
              buf[u] = make_uint4(0, 0, 0, 0);
            } else {
              const uint4* src = reinterpret_cast<const uint4*>(p.ag_src[code >> 26]);
              buf[u] = src[(size_t)(code & 0x3FFFFFF) * sstride + idx % vpr];
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int idx = base + u * CT;
          if (idx < total) dst[(size_t)(idx / vpr) * vpr + idx % vpr] = buf[u];
        }
      }
      fence_proxy_async_global();
      asm volatile("bar.sync 1, %0;" ::"r"(CT));
      if (ct == 0) {
        __threadfence();
        st_release_gpu_s32(&p.ag_flags[g], p.ag_epoch);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p,
            int grid, cudaStream_t stream, bool cooperative = false, int threads = kThreads) {
  auto k = gemm_kernel<BN, STAGES, A_MN, B_MN>;
  constexpr int smem = Smem<BN, STAGES>::TOTAL;
  static bool attr_set[64] = {};  // per template instance and device
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  TORCH_CHECK(dev >= 0 && dev < 64, "gemm: device index");
  if (!attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "cudaFuncSetAttribute(gemm smem)");
    attr_set[dev] = true;
  }
  if (cooperative) {
    CUtensorMap a = ta, b = tb, c = tc;
    Params pp = p;
    void* args[] = {&a, &b, &c, &pp};
    check_cuda(cudaLaunchCooperativeKernel((const void*)k, dim3(grid), dim3(threads), args, smem, stream),
               "gemm cooperative launch");
    return;
  }
  k<<<grid, threads, smem, stream>>>(ta, tb, tc, p);
  check_cuda(cudaGetLastError(), "gemm launch");
}

// ---------------------------------------------------------------------------
// 2-CTA variant (cta_group::2) for large plain GEMMs. A cluster of two CTAs
// owns a 256 x BN output tile: CTA r loads A rows [m0 + 128 r, +128) and B rows
// (output columns) [n0 + r BN/2, +BN/2) with its own plain TMA loads, both
// counted on the leader's (rank 0) full barrier; the leader's MMA warp issues
// 256 x BN x 16 UMMAs that read both CTAs' shared memory, and each CTA's TMEM
// receives its own 128 accumulator rows. Per CTA, a stage holds half the B
// tile of the one-CTA kernel, so the same shared memory keeps more stages in
// flight and each operand byte feeds twice the MMA work.
template <int BN, int STAGES>
struct PairSmem {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + kEpiWarps * 2 * kStageBytesC;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
};

// Bytes CTA ``r`` of a pair loads per K block of tile (tm, tn): a box whose
// first row (A) or column (B) is past the matrix is skipped.
template <int BN, bool A_MN, bool B_MN>
KORE_DEV uint32_t pair_box_bytes(const Params& p, int tm, int tn, int r) {
  const int m0 = tm * 2 * BM + r * BM;
  const int n0 = tn * BN + r * (BN / 2);
  uint32_t b = 0;
  if (!A_MN) {
    b += m0 < p.M ? (uint32_t)(BM * BK * 2) : 0u;
  } else {
#pragma unroll
    for (int j = 0; j < BM / 64; ++j) b += (m0 + 64 * j < p.M) ? 8192u : 0u;
  }
  if (!B_MN) {
    b += n0 < p.N ? (uint32_t)((BN / 2) * BK * 2) : 0u;
  } else {
#pragma unroll
    for (int j = 0; j < BN / 128; ++j) b += (n0 + 64 * j < p.N) ? 8192u : 0u;
  }
  return b;
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, Params p) {
  using S = PairSmem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2] (leader: both CTAs' epilogue warps arrive)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  const int num_m = (p.M + 2 * BM - 1) / (2 * BM);
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, 2 * BN);
  tc_fence_before();
  cluster_sync();   // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
        int tm, tn;
        tile_coords(t, num_m, num_n, tm, tn);
        const int m0 = tm * 2 * BM + (int)rank * BM;
        const int n0 = tn * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1)) { *abort_flag = 1; break; }
          uint8_t* sA = smem + stage * S::STAGE_BYTES;
          uint8_t* sB = sA + S::A_BYTES;
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          // boxes that lie wholly past M or N are not issued (their rows / columns
          // of the accumulator are never stored); the leader expects the bytes
          // both CTAs actually load
          if (rank == 0)
            mbar_arrive_expect_tx(&full_bar[stage], pair_box_bytes<BN, A_MN, B_MN>(p, tm, tn, 0) +
                                                        pair_box_bytes<BN, A_MN, B_MN>(p, tm, tn, 1));
          const int k0 = kb * BK;
          if (!A_MN) {
            if (m0 < p.M) tma_load_2d_pair(sA, &tmA, fb, k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              if (m0 + 64 * j < p.M) tma_load_2d_pair(sA + j * 8192, &tmA, fb, m0 + 64 * j, k0);
          }
          if (!B_MN) {
            if (n0 < p.N) tma_load_2d_pair(sB, &tmB, fb, k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              if (n0 + 64 * j < p.N) tma_load_2d_pair(sB + j * 8192, &tmB, fb, n0 + 64 * j, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    constexpr uint32_t idesc = make_idesc_bf16(2 * BM, BN, A_MN, B_MN);
    if (rank == 0 && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1)) { *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::STAGE_BYTES);
          const uint32_t b_addr = a_addr + S::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad = A_MN ? make_sw128_desc(a_addr + k * 2048, 8192, 1024)
                               : make_sw128_desc(a_addr + k * 32, 16, 1024);
            uint64_t bd = B_MN ? make_sw128_desc(b_addr + k * 2048, 8192, 1024)
                               : make_sw128_desc(b_addr + k * 32, 16, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          umma_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) { *abort_flag = 1; break; }
        umma_commit_pair(&tfull_bar[acc], 0x3);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int lane = threadIdx.x & 31;
    uint8_t* stage_buf = smem + S::EPI_OFF + (warp - 2) * 2 * kStageBytesC;
    const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty_bar[0]), 0),
                                       mapa_shared(smem_u32(&tempty_bar[1]), 0)};
    int buf = 0, it = 0;
    const int CH = p.out_f32 ? 32 : 64;
    for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
      int tm, tn;
      tile_coords(t, num_m, num_n, tm, tn);
      const int m0 = tm * 2 * BM + (int)rank * BM;
      const int n0 = tn * BN;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      ++it;
      if (!mbar_wait(&tfull_bar[acc], acc_phase)) { *abort_flag = 1; break; }
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t t_row = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      for (int c0 = 0; c0 < BN; c0 += CH) {
        if (n0 + c0 >= p.N) break;
        float v[64];
        {
          uint32_t r[32];
          tmem_ld32(t_row + c0, r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
          if (!p.out_f32) {
            tmem_ld32(t_row + c0 + 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) v[32 + i] = __uint_as_float(r[i]) * p.alpha;
          }
        }
        if (row < p.M && (p.accumulate || p.R != nullptr)) {
          const int ncols = min(CH, p.N - (n0 + c0));
          if (p.R != nullptr) {
            const __nv_bfloat16* rp = p.R + (size_t)row * p.ldr + n0 + c0;
#pragma unroll
            for (int j = 0; j < 64; j += 8) {
              if (j >= ncols) break;
              uint4 u = *reinterpret_cast<const uint4*>(rp + j);
              const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
              for (int e = 0; e < 8; ++e) v[j + e] += __bfloat162float(h[e]);
            }
          }
          if (p.accumulate) {
            if (p.out_f32) {
              const float* cp = reinterpret_cast<const float*>(p.C_read) + (size_t)row * p.ldc + n0 + c0;
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                if (j >= ncols) break;
                float4 u = *reinterpret_cast<const float4*>(cp + j);
                v[j] += u.x; v[j + 1] += u.y; v[j + 2] += u.z; v[j + 3] += u.w;
              }
            } else {
              const __nv_bfloat16* cp =
                  reinterpret_cast<const __nv_bfloat16*>(p.C_read) + (size_t)row * p.ldc + n0 + c0;
#pragma unroll
              for (int j = 0; j < 64; j += 8) {
                if (j >= ncols) break;
                uint4 u = *reinterpret_cast<const uint4*>(cp + j);
                const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[j + e] += __bfloat162float(h[e]);
              }
            }
          }
        }
        if (lane == 0) tma_store_wait_read<1>();
        __syncwarp();
        uint8_t* sb = stage_buf + buf * kStageBytesC + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint4 u;
          if (p.out_f32) {
            u.x = __float_as_uint(v[4 * j]);
            u.y = __float_as_uint(v[4 * j + 1]);
            u.z = __float_as_uint(v[4 * j + 2]);
            u.w = __float_as_uint(v[4 * j + 3]);
          } else {
            u.x = pack_bf16(v[8 * j], v[8 * j + 1]);
            u.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
          }
          *reinterpret_cast<uint4*>(sb + ((j ^ (lane & 7)) * 16)) = u;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, stage_buf + buf * kStageBytesC, n0 + c0, m0 + q * 32);
          tma_store_commit();
        }
        buf ^= 1;
      }
      // this CTA's 128 accumulator rows are read: tell the leader's MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
    }
    if (lane == 0) tma_store_wait_all<0>();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();   // the peer's shared memory is no longer read by the leader's MMAs
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const Params& p,
                 int grid, cudaStream_t stream) {
  auto k = gemm_pair_kernel<BN, STAGES, A_MN, B_MN>;
  constexpr int smem = PairSmem<BN, STAGES>::TOTAL;
  static bool attr_set[64] = {};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  TORCH_CHECK(dev >= 0 && dev < 64, "gemm: device index");
  if (!attr_set[dev]) {
    check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
               "cudaFuncSetAttribute(gemm pair smem)");
    attr_set[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CUtensorMap a = ta, b = tb, c = tc;
  Params pp = p;
  check_cuda(cudaLaunchKernelEx(&cfg, k, a, b, c, pp), "gemm pair launch");
}

// Sum of the split-K partials (+ old C when accumulating, + residual) into C.
// One thread per 4 consecutive columns; N % 8 == 0.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int ws_rows, int M, int N,
                                     void* __restrict__ out, int ldc, int out_f32, int accumulate,
                                     const __nv_bfloat16* __restrict__ R, int ldr) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int n4 = N / 4;
  if (i >= (long)M * n4) return;
  const int m = (int)(i / n4), n = (int)(i % n4) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < splits; ++s) {
    const float4 v = *reinterpret_cast<const float4*>(ws + ((size_t)s * ws_rows + m) * N + n);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  if (R != nullptr) {
    const __nv_bfloat162* r = reinterpret_cast<const __nv_bfloat162*>(R + (size_t)m * ldr + n);
    const float2 a = __bfloat1622float2(r[0]), b = __bfloat1622float2(r[1]);
    acc.x += a.x; acc.y += a.y; acc.z += b.x; acc.w += b.y;
  }
  if (out_f32) {
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)m * ldc + n);
    if (accumulate) { const float4 c = *o; acc.x += c.x; acc.y += c.y; acc.z += c.z; acc.w += c.w; }
    *o = acc;
  } else {
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(out) +
                                                          (size_t)m * ldc + n);
    if (accumulate) {
      const float2 a = __bfloat1622float2(o[0]), b = __bfloat1622float2(o[1]);
      acc.x += a.x; acc.y += a.y; acc.z += b.x; acc.w += b.y;
    }
    o[0] = __floats2bfloat162_rn(acc.x, acc.y);
    o[1] = __floats2bfloat162_rn(acc.z, acc.w);
  }
}

// Number of K splits for a problem with `tiles` output tiles: minimises the
// per-SM critical path ceil(tiles*s / sms) * ceil(kblocks / s); 1 when the
// output tiles alone fill the GPU.
int choose_splits(int tiles, int kblocks, int sms) {
  if (tiles >= sms || kblocks < 8) return 1;
  long best = -1;
  int bs = 1;
  for (int s = 1; s <= 16 && s <= kblocks / 4; ++s) {
    const long cost = (long)((tiles * s + sms - 1) / sms) * ((kblocks + s - 1) / s);
    if (best < 0 || cost < best) { best = cost; bs = s; }
  }
  return bs;
}

}  // namespace gemm

// Which kernel large plain GEMMs use: 1 = 2-CTA pairs (cta_group::2), 0 = one CTA per tile.
static int g_gemm_pair_mode = 1;
int64_t gemm_set_pair_mode(int64_t mode) {
  const int old = g_gemm_pair_mode;
  g_gemm_pair_mode = (int)mode;
  return old;
}

// out = alpha * op(a) @ op(b)^T (+ residual) (+ out if accumulate)
//  a: [M,K] if !a_mn else [K,M];  b: [N,K] if !b_mn else [K,N];  out: [M,N] (row stride may exceed N)
void gemm_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, bool a_mn, bool b_mn,
               double alpha, bool accumulate, const c10::optional<at::Tensor>& residual,
               int64_t max_ctas) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm: tensors must be CUDA");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16,
              "gemm: inputs must be bf16");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm: 2-D tensors expected");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1,
              "gemm: inner dimension must be contiguous");
  const bool f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || out.scalar_type() == at::kBFloat16, "gemm: out must be bf16 or fp32");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  const int Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm: K mismatch");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: out shape mismatch");
  // TMA needs 16-byte aligned row strides and contiguous (inner) extents.
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0 && out.stride(0) % (f32 ? 4 : 8) == 0,
              "gemm: row strides must be multiples of 16 bytes");
  TORCH_CHECK(a_mn ? (M % 8 == 0) : (K % 8 == 0), "gemm: A's contiguous extent must be a multiple of 8");
  TORCH_CHECK(b_mn ? (N % 8 == 0) : (K % 8 == 0), "gemm: B's contiguous extent must be a multiple of 8");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  if (K == 0) {
    if (!accumulate) out.zero_();
    if (residual) out.add_(*residual);
    return;
  }
  gemm::Params p;
  p.M = M; p.N = N; p.K = K;
  p.alpha = (float)alpha;
  p.accumulate = accumulate ? 1 : 0;
  p.out_f32 = f32 ? 1 : 0;
  p.C_read = out.data_ptr();
  p.ldc = out.stride(0);
  p.R = nullptr;
  p.ldr = 0;
  p.tiles = nullptr;
  p.C_write = out.data_ptr();
  p.ag_rows = 0;
  p.rs_rows = 0;
  p.rs_rank = 0;
  if (residual) {
    TORCH_CHECK(residual->scalar_type() == at::kBFloat16 && residual->stride(1) == 1 &&
                    residual->size(0) == M && residual->size(1) == N,
                "gemm: residual must be bf16 [M,N] with contiguous rows");
    p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  const int sms = num_sms(a.get_device());
  const int kblocks = (K + 63) / 64;
  bool use256 = N >= 256 && (N % 256 == 0 || N > 1024);
  int splits = 1;
  if (max_ctas <= 0 && M <= 512) {   // skinny (decode-sized) problem: split K over the SMs
    const int t128 = ((M + 127) / 128) * ((N + 127) / 128);
    const int t = use256 ? ((M + 127) / 128) * ((N + 255) / 256) : t128;
    if (t < sms) {
      use256 = false;
      splits = gemm::choose_splits(t128, kblocks, sms);
    }
  }
  const int BN = use256 ? 256 : 128;
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = a_mn ? make_tmap_2d(a.data_ptr(), bf, 2, M, K, a.stride(0), 64, 64)
                        : make_tmap_2d(a.data_ptr(), bf, 2, K, M, a.stride(0), 64, 128);
  cudaStream_t st0 = at::cuda::getCurrentCUDAStream();
  const int pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (g_gemm_pair_mode == 1 && splits == 1 && max_ctas <= 0 && use256 && M > gemm::BM && pair_tiles >= sms) {
    // 2-CTA pairs: each CTA loads half of the 256-column B tile
    CUtensorMap tbp = b_mn ? make_tmap_2d(b.data_ptr(), bf, 2, N, K, b.stride(0), 64, 64)
                           : make_tmap_2d(b.data_ptr(), bf, 2, K, N, b.stride(0), 64, 128);
    CUtensorMap tcp = f32 ? make_tmap_2d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M,
                                         out.stride(0), 32, 32)
                          : make_tmap_2d(out.data_ptr(), bf, 2, N, M, out.stride(0), 64, 32);
    const int grid = std::min(2 * pair_tiles, sms & ~1);
    if (!a_mn && !b_mn) gemm::launch_pair<256, 6, false, false>(ta, tbp, tcp, p, grid, st0);
    else if (!a_mn && b_mn) gemm::launch_pair<256, 6, false, true>(ta, tbp, tcp, p, grid, st0);
    else if (a_mn && !b_mn) gemm::launch_pair<256, 6, true, false>(ta, tbp, tcp, p, grid, st0);
    else gemm::launch_pair<256, 6, true, true>(ta, tbp, tcp, p, grid, st0);
    return;
  }
  CUtensorMap tb = b_mn ? make_tmap_2d(b.data_ptr(), bf, 2, N, K, b.stride(0), 64, 64)
                        : make_tmap_2d(b.data_ptr(), bf, 2, K, N, b.stride(0), 64, BN);
  at::Tensor ws;
  CUtensorMap tc;
  if (splits > 1) {
    // fp32 partial tiles [splits, ws_rows, N]; the reduce kernel applies accumulate / residual
    p.splits = splits;
    p.ws_rows = ((M + 127) / 128) * 128;
    ws = at::empty({(int64_t)splits * p.ws_rows, N}, a.options().dtype(at::kFloat));
    p.out_f32 = 1;
    p.accumulate = 0;
    p.R = nullptr;
    tc = make_tmap_2d(ws.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, (uint64_t)splits * p.ws_rows, N,
                      32, 32);
  } else {
    tc = f32 ? make_tmap_2d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, out.stride(0), 32, 32)
             : make_tmap_2d(out.data_ptr(), bf, 2, N, M, out.stride(0), 64, 32);
  }
  const int tiles = ((M + 127) / 128) * ((N + BN - 1) / BN) * splits;
  int grid = std::min(tiles, sms);
  if (max_ctas > 0) grid = std::min<int>(grid, (int)max_ctas);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define KORE_GEMM_DISPATCH(BN_, ST_)                                              \
  if (!a_mn && !b_mn) gemm::launch<BN_, ST_, false, false>(ta, tb, tc, p, grid, st); \
  else if (!a_mn && b_mn) gemm::launch<BN_, ST_, false, true>(ta, tb, tc, p, grid, st); \
  else if (a_mn && !b_mn) gemm::launch<BN_, ST_, true, false>(ta, tb, tc, p, grid, st); \
  else gemm::launch<BN_, ST_, true, true>(ta, tb, tc, p, grid, st);
  if (use256) {
    KORE_GEMM_DISPATCH(256, 4)
  } else {
    KORE_GEMM_DISPATCH(128, 6)
  }
#undef KORE_GEMM_DISPATCH
  if (splits > 1) {
    const long n = (long)M * (N / 4);
    gemm::splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        ws.data_ptr<float>(), splits, p.ws_rows, M, N, out.data_ptr(), (int)out.stride(0), f32 ? 1 : 0,
        accumulate ? 1 : 0,
        residual ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr,
        residual ? (int)residual->stride(0) : 0);
    check_cuda(cudaGetLastError(), "split-K reduce launch");
    ws.record_stream(at::cuda::getCurrentCUDAStream());
  }
}


// Tensor-parallel GEMMs over peer memory (sequence-parallel layout: the M
// rows are split in W blocks of ``rows`` rows, block i owned by rank i).
//  * all-gather->GEMM (``a_peers`` given): out[M, N] = A . B^T where A's row
//    block i lives on peer i at a_peers[i] (row stride lda). At kernel start
//    the CTAs copy the peers' 64-row groups into the local staging buffer
//    ``stage`` with 16-byte peer loads (each remote row crosses NVLink once)
//    and publish a per-group flag; a tile's producer waits (bounded) for its
//    groups and then TMA-loads A from ``stage``. Tiles start on this rank's
//    own rows, so the first waves overlap the remote copies.
//  * GEMM->reduce-scatter (``rs_peers`` given): out rows are stored into the
//    owner peer's slot buffer (P2P stores): rs_peers[r/rows] +
//    (rank*rows + r%rows) * ldc; the owner then sums its W slots.
void gemm_tp_bf16(const c10::optional<at::Tensor>& a_local, const std::vector<int64_t>& a_peers, int64_t lda,
                  int64_t M, const at::Tensor& b, const c10::optional<at::Tensor>& out,
                  const std::vector<int64_t>& rs_peers, int64_t ldc, int64_t rows, int64_t rank,
                  const c10::optional<at::Tensor>& stage, const c10::optional<at::Tensor>& flags, int64_t epoch) {
  TORCH_CHECK(b.scalar_type() == at::kBFloat16 && b.dim() == 2 && b.stride(1) == 1, "b: bf16 [N, K]");
  const int N = b.size(0), K = b.size(1);
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && rows % 64 == 0 && rows > 0, "tp gemm: N, K % 8 and rows % 64");
  const bool ag = !a_peers.empty();
  const bool rs = !rs_peers.empty();
  TORCH_CHECK(ag || a_local.has_value(), "tp gemm: need a_local or a_peers");
  TORCH_CHECK(rs || out.has_value(), "tp gemm: need out or rs_peers");
  TORCH_CHECK(a_peers.size() <= 8 && rs_peers.size() <= 8, "tp gemm: at most 8 peers");
  c10::cuda::CUDAGuard guard(b.device());
  gemm::Params p;
  p.M = (int)M; p.N = N; p.K = K;
  p.alpha = 1.f;
  p.accumulate = 0;
  p.out_f32 = 0;
  p.R = nullptr; p.ldr = 0;
  p.tiles = nullptr;
  p.C_read = out ? out->data_ptr() : nullptr;
  p.C_write = out ? out->data_ptr() : nullptr;
  p.ldc = rs ? (int)ldc : (int)out->stride(0);
  p.ag_rows = ag ? (int)rows : 0;
  p.rs_rows = rs ? (int)rows : 0;
  p.rs_rank = (int)rank;
  for (int i = 0; i < 8; ++i) { p.rs_out[i] = nullptr; p.ag_src[i] = nullptr; }
  for (size_t i = 0; i < rs_peers.size(); ++i) p.rs_out[i] = reinterpret_cast<void*>(rs_peers[i]);
  p.ag_stage = nullptr; p.ag_flags = nullptr; p.ag_epoch = 0; p.ag_lda = 0; p.ag_rot = 0;
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const bool use256 = N >= 256 && (N % 256 == 0 || N > 1024);
  const int BN = use256 ? 256 : 128;
  CUtensorMap ta;
  if (ag) {
    TORCH_CHECK(stage && flags, "tp gemm: all-gather mode needs a staging buffer and flags");
    TORCH_CHECK(stage->is_cuda() && stage->scalar_type() == at::kBFloat16 && stage->is_contiguous() &&
                    stage->numel() >= M * K, "tp gemm: stage must be contiguous bf16 with >= M*K elements");
    TORCH_CHECK(flags->is_cuda() && flags->scalar_type() == at::kInt && flags->numel() >= M / 64,
                "tp gemm: flags must be int32 with >= M/64 entries");
    TORCH_CHECK(epoch > 0 && lda % 8 == 0 && lda >= K && (int64_t)a_peers.size() * rows == M,
                "tp gemm: epoch > 0, lda % 8, peers * rows == M");
    for (int64_t a : a_peers) TORCH_CHECK(a % 16 == 0, "tp gemm: peer rows must be 16-byte aligned");
    for (size_t i = 0; i < a_peers.size(); ++i) p.ag_src[i] = reinterpret_cast<const void*>(a_peers[i]);
    p.ag_stage = stage->data_ptr();
    p.ag_flags = flags->data_ptr<int>();
    p.ag_epoch = (int)epoch;
    p.ag_lda = (int)lda;
    const int num_m = (int)((M + 127) / 128);
    p.ag_rot = (rows % 128 == 0) ? (int)((rank * rows / 128) % num_m) : 0;
    ta = make_tmap_2d(stage->data_ptr(), bf, 2, K, M, K, 64, 128);
  } else {
    TORCH_CHECK(a_local->stride(1) == 1 && a_local->size(1) == K, "a_local: [M, K]");
    ta = make_tmap_2d(a_local->data_ptr(), bf, 2, K, M, a_local->stride(0), 64, 128);
  }
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), bf, 2, K, N, b.stride(0), 64, BN);
  CUtensorMap tc = rs ? tb : make_tmap_2d(out->data_ptr(), bf, 2, N, M, out->stride(0), 64, 32);
  const int tiles = (int)((M + 127) / 128) * ((N + BN - 1) / BN);
  const int grid = std::min(tiles, num_sms(b.get_device()));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  // all-gather mode: CTAs wait on each other's copies, so they must be co-resident
  if (use256) gemm::launch<256, 4, false, false>(ta, tb, tc, p, grid, st, ag);
  else gemm::launch<128, 6, false, false>(ta, tb, tc, p, grid, st, ag);
}

// Grouped GEMM over experts (MoE): rows of ``a`` are grouped by expert with
// boundaries ``offsets`` (host int64 list, length E+1). For expert e:
//   out[rows_e] (=|+=) a[rows_e] . op(b[e])^T,  b: [E, N, K] (K-major) or [E, K, N] (b_mn)
void gemm_grouped_bf16(const at::Tensor& a, const at::Tensor& b, at::Tensor& out,
                       const std::vector<int64_t>& offsets, bool b_mn, bool accumulate) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16, "grouped gemm: bf16 CUDA tensors");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 3 && out.dim() == 2 && a.stride(1) == 1 && b.is_contiguous() &&
                  out.stride(1) == 1, "grouped gemm: a [M,K], b [E,..] contiguous, out [M,N]");
  const int E = b.size(0);
  TORCH_CHECK((int)offsets.size() == E + 1, "offsets must have E+1 entries");
  const int K = a.size(1);
  const int N = b_mn ? b.size(2) : b.size(1);
  TORCH_CHECK((b_mn ? b.size(1) : b.size(2)) == K, "grouped gemm: K mismatch");
  TORCH_CHECK(out.size(1) == N && out.size(0) == a.size(0), "grouped gemm: out shape");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && a.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "alignment");
  const bool f32 = out.scalar_type() == at::kFloat;
  std::vector<int32_t> tiles;
  for (int e = 0; e < E; ++e)
    for (int64_t m = offsets[e]; m < offsets[e + 1]; m += 128) {
      tiles.push_back(e);
      tiles.push_back((int32_t)m);
      tiles.push_back((int32_t)offsets[e + 1]);
      tiles.push_back(0);
    }
  const int ntm = (int)tiles.size() / 4;
  if (ntm == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  auto tt = at::empty({(int64_t)tiles.size()}, at::TensorOptions().dtype(at::kInt))
                .copy_(at::from_blob(tiles.data(), {(int64_t)tiles.size()}, at::kInt))
                .to(a.device(), /*non_blocking=*/false);
  gemm::Params p;
  p.M = a.size(0); p.N = N; p.K = K;
  p.alpha = 1.f;
  p.accumulate = accumulate ? 1 : 0;
  p.out_f32 = f32 ? 1 : 0;
  p.C_read = out.data_ptr();
  p.C_write = out.data_ptr();
  p.ldc = out.stride(0);
  p.R = nullptr;
  p.ldr = 0;
  p.tiles = reinterpret_cast<const int4*>(tt.data_ptr<int>());
  p.ag_rows = 0;
  p.rs_rows = 0;
  p.rs_rank = 0;
  const bool use256 = N >= 256 && (N % 256 == 0 || N > 1024);
  const int BN = use256 ? 256 : 128;
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), bf, 2, K, a.size(0), a.stride(0), 64, 128);
  CUtensorMap tb = b_mn ? make_tmap_3d(b.data_ptr(), bf, 2, N, K, E, N, (uint64_t)N * K, 64, 64, 1)
                        : make_tmap_3d(b.data_ptr(), bf, 2, K, N, E, K, (uint64_t)N * K, 64, BN, 1);
  CUtensorMap tc = ta;  // unused by the grouped epilogue (masked direct stores)
  // num_m = number of M tiles in the table; tile_coords maps onto it
  p.M = ntm * 128;
  const int tiles_total = ntm * ((N + BN - 1) / BN);
  const int grid = std::min(tiles_total, num_sms(a.get_device()));
  auto cst = at::cuda::getCurrentCUDAStream();
  cudaStream_t st = cst;
  if (use256) {
    if (b_mn) gemm::launch<256, 4, false, true>(ta, tb, tc, p, grid, st);
    else gemm::launch<256, 4, false, false>(ta, tb, tc, p, grid, st);
  } else {
    if (b_mn) gemm::launch<128, 6, false, true>(ta, tb, tc, p, grid, st);
    else gemm::launch<128, 6, false, false>(ta, tb, tc, p, grid, st);
  }
  tt.record_stream(cst);
}

}  // namespace kore

namespace kore {

// Grouped GEMM whose tile table lives on the device (built by moe_plan): no
// host round trip. tiles: int32 [cap * 4] of {expert, first row, row limit, 0};
// ntiles: int32 [1] with the number of valid entries (<= cap).
void gemm_grouped_dev(const at::Tensor& a, const at::Tensor& b, at::Tensor& out, const at::Tensor& tiles,
                      const at::Tensor& ntiles, bool b_mn, bool accumulate) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda() && a.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16, "grouped gemm: bf16 CUDA tensors");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 3 && out.dim() == 2 && a.stride(1) == 1 && b.is_contiguous() &&
                  out.stride(1) == 1, "grouped gemm: a [M,K], b [E,..] contiguous, out [M,N]");
  TORCH_CHECK(tiles.scalar_type() == at::kInt && ntiles.scalar_type() == at::kInt && tiles.is_cuda() &&
                  ntiles.is_cuda(), "grouped gemm: int32 device tile table");
  const int E = b.size(0);
  const int K = a.size(1);
  const int N = b_mn ? b.size(2) : b.size(1);
  TORCH_CHECK((b_mn ? b.size(1) : b.size(2)) == K, "grouped gemm: K mismatch");
  TORCH_CHECK(out.size(1) == N && out.size(0) == a.size(0), "grouped gemm: out shape");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && a.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "alignment");
  const int cap = (int)(tiles.numel() / 4);
  if (cap == 0) return;
  c10::cuda::CUDAGuard guard(a.device());
  const bool f32 = out.scalar_type() == at::kFloat;
  gemm::Params p;
  p.M = cap * 128; p.N = N; p.K = K;
  p.alpha = 1.f;
  p.accumulate = accumulate ? 1 : 0;
  p.out_f32 = f32 ? 1 : 0;
  p.C_read = out.data_ptr();
  p.C_write = out.data_ptr();
  p.ldc = out.stride(0);
  p.R = nullptr; p.ldr = 0;
  p.tiles = reinterpret_cast<const int4*>(tiles.data_ptr<int>());
  p.ntiles_dev = ntiles.data_ptr<int>();
  p.ag_rows = 0; p.rs_rows = 0; p.rs_rank = 0;
  const bool use256 = N >= 256 && (N % 256 == 0 || N > 1024);
  const int BN = use256 ? 256 : 128;
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), bf, 2, K, a.size(0), a.stride(0), 64, 128);
  CUtensorMap tb = b_mn ? make_tmap_3d(b.data_ptr(), bf, 2, N, K, E, N, (uint64_t)N * K, 64, 64, 1)
                        : make_tmap_3d(b.data_ptr(), bf, 2, K, N, E, K, (uint64_t)N * K, 64, BN, 1);
  CUtensorMap tc = ta;   // grouped epilogue stores directly
  const int grid = std::min(cap * ((N + BN - 1) / BN), num_sms(a.get_device()));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (use256) {
    if (b_mn) gemm::launch<256, 4, false, true>(ta, tb, tc, p, grid, st);
    else gemm::launch<256, 4, false, false>(ta, tb, tc, p, grid, st);
  } else {
    if (b_mn) gemm::launch<128, 6, false, true>(ta, tb, tc, p, grid, st);
    else gemm::launch<128, 6, false, false>(ta, tb, tc, p, grid, st);
  }
}

// Grouped GEMM with the expert-parallel dispatch in its prologue (pull
// dispatch): every CTA first copies its share of 64-row groups of the
// receive buffer ``stage`` [cap, K] from the peers' token buffers (addresses
// ``tok_peers``, row stride ``lda``) as ``index`` says (int32 [cap]: peer << 26
// | token row, -1 for pad rows), publishes flags[g] = epoch, and then runs the
// grouped GEMM of gemm_grouped_dev, each tile's producer waiting (bounded) for
// its groups. rows_dev: int32 [1] device count of the receive rows in use (the
// plan's last offset). Cooperative launch: CTAs wait on each other's copies.
void gemm_grouped_dev_pull(at::Tensor& stage, const at::Tensor& b, at::Tensor& out, const at::Tensor& tiles,
                           const at::Tensor& ntiles, const std::vector<int64_t>& tok_peers, int64_t lda,
                           const at::Tensor& index, const at::Tensor& rows_dev, at::Tensor& flags, int64_t epoch,
                           bool b_mn) {
  TORCH_CHECK(stage.is_cuda() && b.is_cuda() && out.is_cuda() && stage.scalar_type() == at::kBFloat16 &&
                  b.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "pull grouped gemm: bf16 CUDA tensors");
  TORCH_CHECK(stage.dim() == 2 && stage.is_contiguous() && b.dim() == 3 && b.is_contiguous() && out.dim() == 2 &&
                  out.stride(1) == 1, "pull grouped gemm: stage [cap, K] contiguous, b [E,..], out [cap, N]");
  TORCH_CHECK(tiles.scalar_type() == at::kInt && ntiles.scalar_type() == at::kInt && index.scalar_type() == at::kInt &&
                  rows_dev.scalar_type() == at::kInt && flags.scalar_type() == at::kInt && tiles.is_cuda() &&
                  ntiles.is_cuda() && index.is_cuda() && rows_dev.is_cuda() && flags.is_cuda(),
              "pull grouped gemm: int32 device tables");
  const int E = b.size(0);
  const int K = stage.size(1);
  const long cap_rows = stage.size(0);
  const int N = b_mn ? b.size(2) : b.size(1);
  TORCH_CHECK((b_mn ? b.size(1) : b.size(2)) == K, "pull grouped gemm: K mismatch");
  TORCH_CHECK(out.size(1) == N && out.size(0) == cap_rows, "pull grouped gemm: out shape");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0 && out.stride(0) % 8 == 0 && lda % 8 == 0 && lda >= K, "alignment");
  TORCH_CHECK(cap_rows % 64 == 0 && index.numel() >= cap_rows && flags.numel() >= cap_rows / 64,
              "pull grouped gemm: cap % 64, index >= cap, flags >= cap / 64");
  TORCH_CHECK(!tok_peers.empty() && tok_peers.size() <= 8 && epoch > 0, "pull grouped gemm: 1..8 peers, epoch > 0");
  for (int64_t a : tok_peers) TORCH_CHECK(a % 16 == 0, "pull grouped gemm: peer rows must be 16-byte aligned");
  const int cap = (int)(tiles.numel() / 4);
  if (cap == 0) return;
  c10::cuda::CUDAGuard guard(stage.device());
  gemm::Params p;
  p.M = cap * 128; p.N = N; p.K = K;
  p.alpha = 1.f;
  p.accumulate = 0;
  p.out_f32 = 0;
  p.C_read = out.data_ptr();
  p.C_write = out.data_ptr();
  p.ldc = out.stride(0);
  p.R = nullptr; p.ldr = 0;
  p.tiles = reinterpret_cast<const int4*>(tiles.data_ptr<int>());
  p.ntiles_dev = ntiles.data_ptr<int>();
  p.ag_rows = 0; p.rs_rows = 0; p.rs_rank = 0;
  for (int i = 0; i < 8; ++i) { p.rs_out[i] = nullptr; p.ag_src[i] = nullptr; }
  for (size_t i = 0; i < tok_peers.size(); ++i) p.ag_src[i] = reinterpret_cast<const void*>(tok_peers[i]);
  p.ag_stage = stage.data_ptr();
  p.ag_flags = flags.data_ptr<int>();
  p.ag_epoch = (int)epoch;
  p.ag_lda = (int)lda;
  p.ag_rot = 0;
  p.ag_index = index.data_ptr<int>();
  p.ag_rows_dev = rows_dev.data_ptr<int>();
  p.ag_cap = (int)cap_rows;
  const bool use256 = N >= 256 && (N % 256 == 0 || N > 1024);
  const int BN = use256 ? 256 : 128;
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = make_tmap_2d(stage.data_ptr(), bf, 2, K, cap_rows, K, 64, 128);
  CUtensorMap tb = b_mn ? make_tmap_3d(b.data_ptr(), bf, 2, N, K, E, N, (uint64_t)N * K, 64, 64, 1)
                        : make_tmap_3d(b.data_ptr(), bf, 2, K, N, E, K, (uint64_t)N * K, 64, BN, 1);
  CUtensorMap tc = ta;   // grouped epilogue stores directly
  const int grid = std::min(cap * ((N + BN - 1) / BN), num_sms(stage.get_device()));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  constexpr int thr = gemm::kThreadsPull;
  if (use256) {
    if (b_mn) gemm::launch<256, 4, false, true>(ta, tb, tc, p, grid, st, true, thr);
    else gemm::launch<256, 4, false, false>(ta, tb, tc, p, grid, st, true, thr);
  } else {
    if (b_mn) gemm::launch<128, 6, false, true>(ta, tb, tc, p, grid, st, true, thr);
    else gemm::launch<128, 6, false, false>(ta, tb, tc, p, grid, st, true, thr);
  }
}

// Per-expert weight gradient over expert-major, 64-row-padded operands:
// out[e] (=|+=) dy[rows_e]^T . x[rows_e], rows_e = [offsets[e], offsets[e+1])
// (device int32, multiples of 64; padding rows are zero). dy [P, M], x [P, N],
// out [E, M, N] (M % 128 == 0). One launch for all experts, no host offsets.
void gemm_grouped_wgrad(const at::Tensor& dy, const at::Tensor& x, at::Tensor& out, const at::Tensor& offsets,
                        bool accumulate) {
  TORCH_CHECK(dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 && dy.is_contiguous() &&
                  x.is_contiguous() && out.is_contiguous() && out.dim() == 3, "grouped wgrad: layouts");
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda(), "grouped wgrad: int32 device offsets");
  const int E = out.size(0), M = out.size(1), N = out.size(2);
  const int P = dy.size(0);
  TORCH_CHECK(dy.size(1) == M && x.size(1) == N && x.size(0) == P && offsets.numel() == E + 1,
              "grouped wgrad: shapes");
  TORCH_CHECK(M % 128 == 0 && N % 64 == 0, "grouped wgrad: M % 128 and N % 64");
  const bool f32 = out.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || out.scalar_type() == at::kBFloat16, "grouped wgrad: out bf16 or fp32");
  if (P == 0 || E == 0) return;
  c10::cuda::CUDAGuard guard(dy.device());
  gemm::Params p;
  p.M = M; p.N = N; p.K = P;
  p.alpha = 1.f;
  p.accumulate = accumulate ? 1 : 0;
  p.out_f32 = f32 ? 1 : 0;
  p.C_read = out.data_ptr();
  p.C_write = out.data_ptr();
  p.ldc = N;
  p.R = nullptr; p.ldr = 0;
  p.tiles = nullptr;
  p.ag_rows = 0; p.rs_rows = 0; p.rs_rank = 0;
  p.wg_offs = offsets.data_ptr<int>();
  p.wg_E = E;
  const bool use256 = N % 256 == 0;
  const int BN = use256 ? 256 : 128;
  auto bf = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap ta = make_tmap_2d(dy.data_ptr(), bf, 2, M, P, M, 64, 64);
  CUtensorMap tb = make_tmap_2d(x.data_ptr(), bf, 2, N, P, N, 64, 64);
  CUtensorMap tc = f32 ? make_tmap_2d(out.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, (uint64_t)E * M, N, 32, 32)
                       : make_tmap_2d(out.data_ptr(), bf, 2, N, (uint64_t)E * M, N, 64, 32);
  const int items = E * (M / 128) * ((N + BN - 1) / BN);
  const int grid = std::min(items, num_sms(dy.get_device()));
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (use256) gemm::launch<256, 4, true, true>(ta, tb, tc, p, grid, st);
  else gemm::launch<128, 6, true, true>(ta, tb, tc, p, grid, st);
}

}  // namespace kore
