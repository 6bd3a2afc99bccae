// K3 / K4: grouped FP8 expert GEMMs on tcgen05 (sm_100a).
//
// Computes, for every expert group g and every token row r of its segment,
//     D[r, m] = sum_k  W_g[m, k] * X[r, k]
// where W_g is the expert's e4m3 weight ([M, K] row-major, the reference's
// ``weight`` layout, inference/ops.py:15-28) with one fp32 ``weight_scale_inv``
// per 128x128 block, and X is the token activation held as two e4m3 terms that
// share one fp32 scale per (row, 128-wide K block): x ~= (hi + lo) * sx.
//
// Mapping to the tensor core ("swap AB"): the weight tile is the 128-row A
// operand (M = 128 output features), the tokens are the N operand (N = 32..128
// tokens, a multiple of 32), so decode-sized groups of a few tokens waste
// little work. For every 128-wide K block the MMA writes a fresh fp32 partial
// (hi and lo accumulate into the same partial) into one of two TMEM buffers;
// the epilogue warps read it back and promote it into fp32 registers:
//     acc[m, r] += partial[m, r] * sw[mb, kb] * sx[r, kb]
// which is the reference's fp32 dequant-then-matmul (inference/ops.py:40-44)
// reassociated per 128-K block.
//
// Two instantiations:
//   NB = 2  gate/up: W_gate and W_up tiles of the same 128 features share the
//           token tile; the epilogue forms h = silu(g) * u with the reference's
//           bf16 roundings (inference/ops.py:186-192) and writes h back as a
//           hi/lo e4m3 pair with one scale per (row, 128 features) — the
//           down GEMM's activation format.
//   NB = 1  down: the epilogue writes y = bf16(acc) per permuted row.
//
// Warp roles (320 threads, one CTA per SM, persistent over work units):
//   warp 0      TMA producer (one thread)
//   warp 1      TMEM allocator + MMA issuer (one thread)
//   warps 2-9   epilogue: warp w reads TMEM lane quadrant (w % 4) and a
//               64-column half ((w - 2) / 4) of every accumulator.
// (Registers are split over the SM's four 16K-register sub-partitions, so
// 10 warps leave up to 168 registers per thread for the accumulators.)
// Work unit = (group, 128-feature tile, 128-token tile); units are ordered
// group-major, then feature tile, then token tile, so CTAs that work on the
// token tiles of one feature tile read the same weight tile close in time.
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace gg {
constexpr int BM = 128;   // weight rows (output features) per tile
constexpr int BN = 128;   // max tokens per tile
constexpr int BK = 128;   // K bytes per stage
constexpr int SUB = 32;   // token rows per activation TMA box
constexpr int NUM_EPI_WARPS = 8;
constexpr int EPI_COLS = BN * 4 / NUM_EPI_WARPS;  // accumulator columns per epilogue warp
constexpr int NUM_THREADS = (2 + NUM_EPI_WARPS) * 32;
constexpr int MAX_GROUPS = 264;

template <int NB>
struct Cfg {
  static constexpr int STAGES = NB == 2 ? 3 : 4;
  static constexpr int XH_OFF = NB * BM * BK;
  static constexpr int XL_OFF = XH_OFF + BN * BK;
  static constexpr int SX_OFF = XL_OFF + BN * BK;
  static constexpr int STAGE_BYTES = ((SX_OFF + BN * 4 + 1023) / 1024) * 1024;
  static constexpr int TMEM_COLS = NB == 2 ? 512 : 256;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  // barriers: full[S], empty[S], tfull[2], tempty[2], done
  static constexpr int MISC_OFF = BAR_OFF + 8 * (2 * STAGES + 5);
  static constexpr int TABLE_OFF = ((MISC_OFF + 16 + 15) / 16) * 16;
  static constexpr int RED_OFF = TABLE_OFF + 4 * 4 * MAX_GROUPS;
  static constexpr int SMEM_BYTES = RED_OFF + 4 * 4 * 32 * 4 + 1024;  // + alignment slack
};

// unit -> (group, feature tile, token tile)
__device__ __forceinline__ void decode_unit(int u, int n_groups, const int* ustart, const int* counts, int& g,
                                            int& mt, int& nt, int& ntiles) {
  int lo = 0, hi = n_groups;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ustart[mid] <= u) lo = mid; else hi = mid;
  }
  g = lo;
  ntiles = (counts[g] + BN - 1) / BN;
  const int local = u - ustart[g];
  mt = local / ntiles;
  nt = local - mt * ntiles;
}

__device__ __forceinline__ float silu_f32(float x) { return x / (1.0f + expf(-x)); }

template <int NB>
__global__ void __launch_bounds__(NUM_THREADS, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_sx,
                    const GemmParams p) {
  using C = Cfg<NB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done_bar = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);
  int* s_ustart = reinterpret_cast<int*>(smem + C::TABLE_OFF);
  int* s_counts = s_ustart + MAX_GROUPS;
  int* s_rows = s_counts + MAX_GROUPS;
  int* s_slot = s_rows + MAX_GROUPS;
  float* s_red = reinterpret_cast<float*>(smem + C::RED_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NG = p.n_groups;

  for (int i = threadIdx.x; i <= NG; i += blockDim.x) {
    s_ustart[i] = p.unit_start[i];
    if (i < NG) {
      s_counts[i] = p.counts[i];
      s_rows[i] = p.row_start[i];
      s_slot[i] = p.slot_of[i];
    }
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + NUM_EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], NUM_EPI_WARPS);
    }
    mbar_init(done_bar, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w0);
    if (NB == 2) prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_sx);
  }
  if (warp == 1) tmem_alloc(s_tmem, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = *s_tmem;
  const int total_units = s_ustart[NG];
  const int n_kb = p.K / BK;
  const int mtiles = p.M / BM;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int g, mt, nt, ntiles;
        decode_unit(u, NG, s_ustart, s_counts, g, mt, nt, ntiles);
        const int slot = s_slot[g];
        if (slot < 0 || slot >= p.n_slots) {
          atomicCAS(p.status, 0, kDevBadSlot);
          *s_abort = 1;
          break;
        }
        const int col0 = nt * BN;
        const int ncols = min(BN, s_counts[g] - col0);
        const int nsub = (ncols + SUB - 1) / SUB;
        const int row0 = s_rows[g] + col0;
        const int wrow = slot * p.M + mt * BM;
        const uint32_t bytes = NB * BM * BK + 2 * nsub * SUB * BK + BN * 4;
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kDevTimeoutProducer, s_abort)) { ok = false; break; }
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(st, &tm_w0, &full[stage], kb * BK, wrow, pol_w);
          if (NB == 2) tma_load_2d(st + BM * BK, &tm_w1, &full[stage], kb * BK, wrow, pol_w);
          for (int s = 0; s < nsub; ++s) {
            tma_load_2d(st + C::XH_OFF + s * SUB * BK, &tm_x, &full[stage], kb * BK, row0 + s * SUB, pol_x);
            tma_load_2d(st + C::XL_OFF + s * SUB * BK, &tm_x, &full[stage], kb * BK, p.P + row0 + s * SUB, pol_x);
          }
          tma_load_2d(st + C::SX_OFF, &tm_sx, &full[stage], row0, kb, pol_x);
          ++issued;
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: the copies of the last min(issued, STAGES) stages must have
      // landed before the CTA may exit (they normally have been consumed).
      const int n_drain = issued < C::STAGES ? issued : C::STAGES;
      for (int i = 0; i < n_drain; ++i) {
        if (--stage < 0) { stage = C::STAGES - 1; phase ^= 1; }
        mbar_wait(&full[stage], phase, p.status, kDevTimeoutProducer, s_abort);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int tb = 0;
      uint32_t tphase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int g, mt, nt, ntiles;
        decode_unit(u, NG, s_ustart, s_counts, g, mt, nt, ntiles);
        const int ncols = min(BN, s_counts[g] - nt * BN);
        const int N = ((ncols + SUB - 1) / SUB) * SUB;
        const uint32_t idesc = idesc_e4m3(BM, N);
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&tempty[tb], tphase ^ 1, p.status, kDevTimeoutMma, s_abort)) { ok = false; break; }
          if (!mbar_wait(&full[stage], phase, p.status, kDevTimeoutMma, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sbase = smem_u32(smem + stage * C::STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            const uint32_t d = tmem_base + tb * (NB * BN) + j * BN;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t xoff = h ? C::XL_OFF : C::XH_OFF;
#pragma unroll
              for (int kk = 0; kk < BK / 32; ++kk) {
                mma_f8f6f4(d, umma_desc_sw128(sbase + j * BM * BK + kk * 32),
                           umma_desc_sw128(sbase + xoff + kk * 32), idesc, (h | kk) != 0);
              }
            }
          }
          mma_commit(&empty[stage]);
          mma_commit(&tfull[tb]);
          if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
          tb ^= 1;
          if (tb == 0) tphase ^= 1;
        }
      }
      // All MMAs issued by this thread complete before TMEM is released.
      mma_commit(done_bar);
      mbar_wait(done_bar, 0, p.status, kDevTimeoutMma, s_abort);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp w reads TMEM lane quadrant (w % 4) and the 64-column half
    // ((w - 2) / 4) of every accumulator.
    const int quad = warp & 3;
    const int ch = (warp - 2) >> 2;
    const int c0 = ch * EPI_COLS;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int stage = 0;
    uint32_t phase = 0;
    int tb = 0;
    uint32_t tphase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      int g, mt, nt, ntiles;
      decode_unit(u, NG, s_ustart, s_counts, g, mt, nt, ntiles);
      const int slot = s_slot[g];
      const int ncols = min(BN, s_counts[g] - nt * BN);
      const int nvalid = max(0, min(EPI_COLS, ncols - c0));  // valid columns of this warp
      // Weight block scales of this unit's 128-row tile, one per K block:
      // lane i holds kb = i and kb = 32 + i.
      float swr[NB][2];
      {
        const bool slot_ok = slot >= 0 && slot < p.n_slots;  // the producer reports a bad slot
        const size_t base = (static_cast<size_t>(slot_ok ? slot : 0) * mtiles + mt) * n_kb;
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const float* ws = j == 0 ? p.wscale0 : p.wscale1;
          swr[j][0] = slot_ok && lane < n_kb ? __ldg(ws + base + lane) : 0.f;
          swr[j][1] = slot_ok && 32 + lane < n_kb ? __ldg(ws + base + 32 + lane) : 0.f;
        }
      }
      float acc[NB][EPI_COLS];
#pragma unroll
      for (int j = 0; j < NB; ++j)
#pragma unroll
        for (int i = 0; i < EPI_COLS; ++i) acc[j][i] = 0.f;

      for (int kb = 0; kb < n_kb; ++kb) {
        if (!mbar_wait(&tfull[tb], tphase, p.status, kDevTimeoutEpilogue, s_abort)) { ok = false; break; }
        if (!mbar_wait(&full[stage], phase, p.status, kDevTimeoutEpilogue, s_abort)) { ok = false; break; }
        tc_fence_after();
        const float4* sx4 = reinterpret_cast<const float4*>(smem + stage * C::STAGE_BYTES + C::SX_OFF) + (c0 >> 2);
        float swj[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j) swj[j] = __shfl_sync(0xffffffffu, swr[j][kb >> 5], kb & 31);
#pragma unroll
        for (int q8 = 0; q8 < EPI_COLS / 8; ++q8) {
          if (q8 * 8 < nvalid) {  // warp-uniform
            const float4 s0 = sx4[q8 * 2], s1 = sx4[q8 * 2 + 1];
            const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int j = 0; j < NB; ++j) {
              float part[8];
              tmem_ld8(tmem_base + lane_base + tb * (NB * BN) + j * BN + c0 + q8 * 8, part);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[j][q8 * 8 + i] = fmaf(part[i], sv[i] * swj[j], acc[j][q8 * 8 + i]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&tempty[tb]);
          mbar_arrive(&empty[stage]);
        }
        if (++stage == C::STAGES) { stage = 0; phase ^= 1; }
        tb ^= 1;
        if (tb == 0) tphase ^= 1;
      }
      // A warp that gave up still takes this unit's named barriers below, so
      // the other warps of its column half are not left waiting.
      const int nstore = ok ? nvalid : 0;

      const int row_base = s_rows[g] + nt * BN + c0;
      const int feat = mt * BM + quad * 32 + lane;
      if constexpr (NB == 1) {
#pragma unroll
        for (int i = 0; i < EPI_COLS; ++i) {
          if (i < nstore) p.y[static_cast<size_t>(row_base + i) * p.M + feat] = __float2bfloat16_rn(acc[0][i]);
        }
      } else {
        // h = bf16(bf16(silu(bf16(g))) * bf16(u)), then one scale per token
        // over this tile's 128 features (4 warps x 32 lanes).
#pragma unroll
        for (int i = 0; i < EPI_COLS; ++i) {
          const float gt = bf16_round(silu_f32(bf16_round(acc[0][i])));
          acc[0][i] = bf16_round(gt * bf16_round(acc[1][i]));
        }
#pragma unroll
        for (int sc = 0; sc < EPI_COLS / 32; ++sc) {
          if (sc * 32 < nstore) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = fabsf(acc[0][sc * 32 + i]);
            // Transpose-reduce: afterwards lane l holds the warp max of column l.
#pragma unroll
            for (int w = 16; w >= 1; w >>= 1) {
              const bool upper = (lane & w) != 0;
#pragma unroll
              for (int i = 0; i < w; ++i) {
                const float send = upper ? v[i] : v[i + w];
                const float keep = upper ? v[i + w] : v[i];
                v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, w));
              }
            }
            s_red[((ch * 2 + sc) * 4 + quad) * 32 + lane] = v[0];
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + ch) : "memory");
        uint8_t* hq_hi = p.hq;
        uint8_t* hq_lo = p.hq + static_cast<size_t>(p.P) * p.M;
#pragma unroll
        for (int sc = 0; sc < EPI_COLS / 32; ++sc) {
          if (sc * 32 < nstore) {
            float amax = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) amax = fmaxf(amax, s_red[((ch * 2 + sc) * 4 + q) * 32 + lane]);
            const float inv = amax > 0.f ? 448.f / amax : 0.f;
            const float scale = amax / 448.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float q = acc[0][sc * 32 + i] * __shfl_sync(0xffffffffu, inv, i);
              if (sc * 32 + i < nstore) {
                const uint16_t hi2 = f32x2_to_e4m3x2(q, 0.f);
                const float hif = e4m3_to_f32(static_cast<uint8_t>(hi2 & 0xff));
                const uint16_t lo2 = f32x2_to_e4m3x2(q - hif, 0.f);
                const size_t off = static_cast<size_t>(row_base + sc * 32 + i) * p.M + feat;
                hq_hi[off] = static_cast<uint8_t>(hi2 & 0xff);
                hq_lo[off] = static_cast<uint8_t>(lo2 & 0xff);
              }
            }
            if (quad == 0 && sc * 32 + lane < nstore)
              p.hs[static_cast<size_t>(mt) * p.P + row_base + sc * 32 + lane] = scale;
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + ch) : "memory");
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace gg

int gemm_smem_bytes(int nb) { return nb == 2 ? gg::Cfg<2>::SMEM_BYTES : gg::Cfg<1>::SMEM_BYTES; }

cudaError_t launch_grouped_gemm(int nb, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                                const CUtensorMap& sx, const GemmParams& p, int grid, cudaStream_t stream) {
  if (p.n_groups > gg::MAX_GROUPS - 1) return cudaErrorInvalidValue;
  if (nb == 2) {
    static bool attr = false;
    if (!attr) {
      cudaError_t e = cudaFuncSetAttribute(gg::grouped_gemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gg::Cfg<2>::SMEM_BYTES);
      if (e != cudaSuccess) return e;
      attr = true;
    }
    gg::grouped_gemm_kernel<2><<<grid, gg::NUM_THREADS, gg::Cfg<2>::SMEM_BYTES, stream>>>(w0, w1, x, sx, p);
  } else {
    static bool attr = false;
    if (!attr) {
      cudaError_t e = cudaFuncSetAttribute(gg::grouped_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           gg::Cfg<1>::SMEM_BYTES);
      if (e != cudaSuccess) return e;
      attr = true;
    }
    gg::grouped_gemm_kernel<1><<<grid, gg::NUM_THREADS, gg::Cfg<1>::SMEM_BYTES, stream>>>(w0, w0, x, sx, p);
  }
  return cudaGetLastError();
}

}  // namespace dsmoe
