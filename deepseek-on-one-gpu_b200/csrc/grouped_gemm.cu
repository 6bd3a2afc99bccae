// K3 / K4: grouped FP8 expert GEMMs on tcgen05 (sm_100a).
//
// Computes, for every expert group g, every token row r of its segment and
// every output feature m of one or two stacked weight matrices,
//     Y[r, m] = bf16( sum_k  W_g[m, k] * X[r, k] )
// where W_g is the expert's e4m3 weight ([M, K] row-major, the reference's
// ``weight`` layout, inference/ops.py:15-28) with one fp32 ``weight_scale_inv``
// per 128x128 block, and X is the token activation held as two e4m3 terms that
// share one fp32 scale per row: x ~= (hi + lo) * sx[r].
//
// Mapping to the tensor core ("swap AB"): the weight tile is the 128-row A
// operand (M = 128 output features), the tokens are the N operand, so
// decode-sized groups of a few tokens waste little work. For every 128-wide K
// block the MMA writes a fresh fp32 partial of W*hi + W*lo into one of NBUF
// TMEM buffers (tiles of up to 128 tokens put hi and lo side by side in one
// MMA of N = 2 * tile; wider tiles accumulate hi then lo along K);
// the epilogue warps read it back and promote it with the block's weight scale:
//     acc[m, r] += sw[mb, kb] * partial[m, r]
// and finally write bf16(acc * sx[r]) — the reference's fp32
// dequant-then-matmul (inference/ops.py:40-44) reassociated per 128-K block,
// rounded to bf16 like the reference's fp8_linear output.
//
// Gate/up: the gate and up weights are two matrices of one launch (feature
// tiles 0..F/128-1 read the gate bank, the rest the up bank) and the output
// row is [g | u] (2F wide); swiglu_quant.cu forms h = silu(g) * u.
//
// Warp roles (608 threads, one CTA per SM, persistent over work units):
//   warp 0      TMA producer (one thread)
//   warp 1      TMEM allocator + MMA issuer for even K steps (one thread)
//   warps 2-17  epilogue: warp w reads TMEM lane quadrant (w % 4) and the
//               column group ((w - 2) / 4) of BN / 4 accumulator columns.
//   warp 18     MMA issuer for odd K steps (one thread)
// Two issuers: a thread that waits on an mbarrier between its MMA batches
// leaves the tensor pipe idle for a few hundred cycles each time; with the
// K steps split by parity one issuer's MMAs run while the other waits. Every
// K step writes its own TMEM buffer and smem stage, so the two streams are
// independent; each issuer commits only its own MMAs.
// The SM's register file is split over four 16K-register sub-partitions and
// 19 warps put 5 warps on some of them, so the kernel is capped at 96
// registers per thread.
// Activation tiles are one TMA box of BN rows per term (hi, lo); groups of at
// most 64 tokens use 32-row boxes instead so decode steps do not pull BN rows.
// Work unit = (group, 128-feature tile, BN-token tile); units are ordered
// group-major, then feature tile, then token tile.
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace gg {
constexpr int BM = 128;   // weight rows (output features) per tile
constexpr int BK = 128;   // K bytes per stage
constexpr int SUB = 32;   // token rows per small activation TMA box
constexpr int NUM_EPI_WARPS = 16;
constexpr int NUM_MMA_ISSUERS = 2;
constexpr int NUM_THREADS = (2 + NUM_EPI_WARPS + 1) * 32;
constexpr int ISSUER_B_WARP = 2 + NUM_EPI_WARPS;
constexpr int MAX_GROUPS = 264;

template <int BN_, int STAGES_, int NBUF_, bool NCAT_>
struct Cfg {
  static constexpr int BN = BN_;                  // max tokens per tile
  static constexpr int STAGES = STAGES_;
  static constexpr int NBUF = NBUF_;              // TMEM accumulator buffers (MMA runs NBUF-1 K steps ahead)
  // hi and lo rows are adjacent in shared memory; for tiles of up to 128
  // tokens one MMA covers both (N = 2 * BN, columns [0,BN) hi, [BN,2BN) lo),
  // halving the MMA count; wider tiles accumulate hi then lo along K.
  static constexpr bool NCAT = NCAT_;
  static constexpr int TCOLS = NCAT ? 2 * BN : BN;  // TMEM columns per buffer
  static constexpr int EPI_COLS = BN / 4;         // accumulator columns per epilogue warp
  static constexpr int CHUNK = EPI_COLS % 16 ? 8 : 16;  // columns per TMEM load
  static constexpr int XH_OFF = BM * BK;
  static constexpr int XL_OFF = XH_OFF + BN * BK;
  static constexpr int STAGE_BYTES = XL_OFF + BN * BK;  // multiple of 1024 for BN % 8 == 0
  static constexpr int TMEM_COLS = NBUF * TCOLS <= 32 ? 32 : NBUF * TCOLS <= 64 ? 64 : NBUF * TCOLS <= 128 ? 128
                                   : NBUF * TCOLS <= 256 ? 256 : 512;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  // barriers: full[S], empty[S], tfull[NBUF], tempty[NBUF], done
  static constexpr int NUM_BARS = 2 * STAGES + 2 * NBUF + 1;
  static constexpr int MISC_OFF = BAR_OFF + 8 * NUM_BARS;
  static constexpr int TABLE_OFF = ((MISC_OFF + 16 + 15) / 16) * 16;
  // Of the per-group tables only the unit prefix sums (searched at every
  // unit start) live in shared memory; the rest is read from global memory
  // (L1-cached), so that shared memory goes to the stage ring.
  static constexpr int SMEM_BYTES = TABLE_OFF + 4 * MAX_GROUPS + 1024;  // + alignment slack
  static_assert(BN % 32 == 0 && BN <= 256 && EPI_COLS % CHUNK == 0 && NBUF * TCOLS <= 512 &&
                    (!NCAT || 2 * BN <= 256), "tile shape");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// unit -> (group, feature tile, token tile)
template <int BN>
__device__ __forceinline__ void decode_unit(int u, int n_groups, const int* ustart, const int* counts, int& g,
                                            int& mt, int& nt) {
  int lo = 0, hi = n_groups;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ustart[mid] <= u) lo = mid; else hi = mid;
  }
  g = lo;
  const int ntiles = (counts[g] + BN - 1) / BN;
  const int local = u - ustart[g];
  mt = local / ntiles;
  nt = local - mt * ntiles;
}

template <int BN_, int STAGES_, int NBUF_, bool NCAT_>
__global__ void __maxnreg__(96)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_x32,
                    const GemmParams p) {
  using C = Cfg<BN_, STAGES_, NBUF_, NCAT_>;
  constexpr int BN = C::BN;
  constexpr int STAGES = C::STAGES;
  constexpr int NBUF = C::NBUF;
  constexpr int EPI_COLS = C::EPI_COLS;
  constexpr int CHUNK = C::CHUNK;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NBUF;
  uint64_t* done_bar = tempty + NBUF;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);
  int* s_ustart = reinterpret_cast<int*>(smem + C::TABLE_OFF);
  const int* __restrict__ s_counts = p.counts;
  const int* __restrict__ s_rows = p.row_start;
  const int* __restrict__ s_slot = p.slot_of;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NG = p.n_groups;

  for (int i = threadIdx.x; i <= NG; i += blockDim.x) s_ustart[i] = p.unit_start[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], NUM_EPI_WARPS);
    }
    mbar_init(done_bar, NUM_MMA_ISSUERS);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w0);
    if (p.n_mat == 2) prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_x32);
  }
  if (warp == 1) tmem_alloc(s_tmem, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem_base = *s_tmem;
  const int total_units = s_ustart[NG];
  const int n_kb = p.K / BK;
  // 128-row tiles per matrix; a ragged last tile (single-slot linear layers
  // such as 576 outputs) reads zero-filled rows past the end of the weight
  // and stores only rows < M.
  const int mt_per_mat = (p.M + BM - 1) / BM;

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
        int g, mt, nt;
        decode_unit<BN>(u, NG, s_ustart, s_counts, g, mt, nt);
        const int slot = s_slot[g];
        if (slot < 0 || slot >= p.n_slots) {
          atomicCAS(p.status, 0, kDevBadSlot);
          *s_abort = 1;
          break;
        }
        const int mat = mt >= mt_per_mat;
        const CUtensorMap* tw = mat ? &tm_w1 : &tm_w0;
        const int col0 = nt * BN;
        const int ncols = min(BN, s_counts[g] - col0);
        const int nsub = (ncols + SUB - 1) / SUB;
        // A few 32-row boxes beat one big box; four or more cost more than the
        // rows they save (a 128-token tile as 4 boxes: +8% kernel time).
        const bool small = BN == SUB || (nsub * SUB < BN && nsub <= 2);
        const int row0 = s_rows[g] + col0;
        const int wrow = slot * p.M + (mt - mat * mt_per_mat) * BM;
        const uint32_t bytes = BM * BK + 2 * (small ? nsub * SUB : BN) * BK;
        for (int kb = 0; kb < n_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.status, kDevTimeoutProducer, s_abort)) { ok = false; break; }
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(st, tw, &full[stage], kb * BK, wrow, pol_w);
          if (small) {
            for (int s = 0; s < nsub; ++s) {
              tma_load_2d(st + C::XH_OFF + s * SUB * BK, &tm_x32, &full[stage], kb * BK, row0 + s * SUB, pol_x);
              tma_load_2d(st + C::XL_OFF + s * SUB * BK, &tm_x32, &full[stage], kb * BK, p.P + row0 + s * SUB,
                          pol_x);
            }
          } else {
            tma_load_2d(st + C::XH_OFF, &tm_x, &full[stage], kb * BK, row0, pol_x);
            tma_load_2d(st + C::XL_OFF, &tm_x, &full[stage], kb * BK, p.P + row0, pol_x);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: the copies of the last issued stages must have landed before
      // the CTA may exit (normally they were consumed already).
      const int n_drain = issued < STAGES ? issued : STAGES;
      for (int i = 0; i < n_drain; ++i) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        mbar_wait(&full[stage], phase, p.status, kDevTimeoutProducer, s_abort);
      }
    }
  } else if (warp == 1 || warp == ISSUER_B_WARP) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const int me = warp == 1 ? 0 : 1;  // issues the K steps of this parity
      int step = 0;
      int stage = 0;
      uint32_t phase = 0;
      int tb = 0;
      uint32_t tphase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        int g, mt, nt;
        decode_unit<BN>(u, NG, s_ustart, s_counts, g, mt, nt);
        const int ncols = min(BN, s_counts[g] - nt * BN);
        const int N = C::NCAT ? 2 * BN : (ncols + 15) & ~15;
        const uint32_t idesc = idesc_e4m3(BM, N);
        for (int kb = 0; kb < n_kb; ++kb, ++step) {
          if ((step & 1) != me) {  // the other issuer's step: only advance the rings
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
            if (++tb == NBUF) { tb = 0; tphase ^= 1; }
            continue;
          }
          if (!mbar_wait(&tempty[tb], tphase ^ 1, p.status, kDevTimeoutMma, s_abort)) { ok = false; break; }
          if (!mbar_wait(&full[stage], phase, p.status, kDevTimeoutMma, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sbase = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t d = tmem_base + tb * C::TCOLS;
          if constexpr (C::NCAT) {
#pragma unroll
            for (int kk = 0; kk < BK / 32; ++kk)
              mma_f8f6f4(d, umma_desc_sw128(sbase + kk * 32), umma_desc_sw128(sbase + C::XH_OFF + kk * 32), idesc,
                         kk != 0);
          } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t xoff = h ? C::XL_OFF : C::XH_OFF;
#pragma unroll
              for (int kk = 0; kk < BK / 32; ++kk)
                mma_f8f6f4(d, umma_desc_sw128(sbase + kk * 32), umma_desc_sw128(sbase + xoff + kk * 32), idesc,
                           (h | kk) != 0);
            }
          }
          mma_commit(&empty[stage]);
          mma_commit(&tfull[tb]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
          if (++tb == NBUF) { tb = 0; tphase ^= 1; }
        }
      }
      // All MMAs of both issuers complete before TMEM is released (the
      // barrier's first phase needs one commit from each).
      mma_commit(done_bar);
      mbar_wait(done_bar, 0, p.status, kDevTimeoutMma, s_abort);
    }
  } else if (warp >= 2 && warp < 2 + NUM_EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int cg = (warp - 2) >> 2;
    const int c0 = cg * EPI_COLS;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int out_ld = p.n_mat * p.M;
    int tb = 0;
    uint32_t tphase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      int g, mt, nt;
      decode_unit<BN>(u, NG, s_ustart, s_counts, g, mt, nt);
      const int slot = s_slot[g];
      const int ncols = min(BN, s_counts[g] - nt * BN);
      const int nvalid = max(0, min(EPI_COLS, ncols - c0));  // valid columns of this warp
      const int mat = mt >= mt_per_mat;
      // Weight block scales of this unit's 128-row tile, one per K block, in
      // two 32-block windows: lane i holds kb = 32w + i of window w in
      // register w % 2; entering window w refills the other register with
      // window w + 1, 32 K steps before it is needed.
      const bool slot_ok = slot >= 0 && slot < p.n_slots;  // the producer reports a bad slot
      const float* wsc = (mat ? p.wscale1 : p.wscale0) +
                         (static_cast<size_t>(slot_ok ? slot : 0) * mt_per_mat + (mt - mat * mt_per_mat)) * n_kb;
      float swr0 = slot_ok && lane < n_kb ? __ldg(wsc + lane) : 0.f;
      float swr1 = slot_ok && 32 + lane < n_kb ? __ldg(wsc + 32 + lane) : 0.f;
      // Per-row activation scales of this warp's columns (lane i holds column
      // i and 32 + i), loaded now so that the latency hides behind the K loop.
      const int row_base = s_rows[g] + nt * BN + c0;
      const float sxa = lane < nvalid ? __ldg(p.sx + row_base + lane) : 0.f;
      const float sxb = 32 + lane < nvalid ? __ldg(p.sx + row_base + 32 + lane) : 0.f;
      float acc[EPI_COLS];
#pragma unroll
      for (int i = 0; i < EPI_COLS; ++i) acc[i] = 0.f;

      for (int kb = 0; kb < n_kb; ++kb) {
        if (!mbar_wait(&tfull[tb], tphase, p.status, kDevTimeoutEpilogue, s_abort)) { ok = false; break; }
        tc_fence_after();
        if ((kb & 31) == 0 && kb >= 32) {
          const int nk = kb + 32 + lane;
          const float v = slot_ok && nk < n_kb ? __ldg(wsc + nk) : 0.f;
          if ((kb >> 5) & 1) swr0 = v; else swr1 = v;
        }
        const float sw = __shfl_sync(0xffffffffu, ((kb >> 5) & 1) ? swr1 : swr0, kb & 31);
#pragma unroll
        for (int q = 0; q < EPI_COLS / CHUNK; ++q) {
          if (q * CHUNK < nvalid) {  // warp-uniform
            const uint32_t ta = tmem_base + lane_base + tb * C::TCOLS + c0 + q * CHUNK;
            float part[CHUNK];
            if constexpr (CHUNK == 16) tmem_ld16(ta, part);
            else tmem_ld8(ta, part);
            if constexpr (C::NCAT) {
              float lo[CHUNK];
              if constexpr (CHUNK == 16) tmem_ld16(ta + BN, lo);
              else tmem_ld8(ta + BN, lo);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < CHUNK; ++i) part[i] += lo[i];
            } else {
              tmem_ld_wait();
            }
            // Packed fp32x2 FMAs: half the issue slots of scalar fmaf, same
            // rounding (-2% kernel time at T=4096, where the GEMM runs at
            // the power cap).
#pragma unroll
            for (int i = 0; i < CHUNK; i += 2)
              fma2(acc[q * CHUNK + i], acc[q * CHUNK + i + 1], part[i], part[i + 1], sw);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[tb]);
        if (++tb == NBUF) { tb = 0; tphase ^= 1; }
      }
      if (!ok) break;
      // Stores of bf16 pairs: for tokens i and i+1, an even lane writes
      // features (lane, lane+1) of token i and its odd neighbour features
      // (lane-1, lane) of token i+1; one shuffle exchanges the halves.
      const int odd = lane & 1;
      const int row_in_mat = (mt - mat * mt_per_mat) * BM + quad * 32 + (lane & ~1);  // the pair's first row
      const bool row_ok = row_in_mat < p.M;  // M is even: the pair is inside or outside together
      __nv_bfloat16* ybase = p.y + mat * p.M + row_in_mat;
#pragma unroll
      for (int i = 0; i < EPI_COLS; i += 2) {
        const float s0 = __shfl_sync(0xffffffffu, i < 32 ? sxa : sxb, i & 31);
        const float s1 = __shfl_sync(0xffffffffu, i + 1 < 32 ? sxa : sxb, (i + 1) & 31);
        const __nv_bfloat16 v0 = __float2bfloat16_rn(acc[i] * s0);
        const __nv_bfloat16 v1 = __float2bfloat16_rn(acc[i + 1] * s1);
        const unsigned short mine = __bfloat16_as_ushort(odd ? v1 : v0);
        const unsigned short other = static_cast<unsigned short>(
            __shfl_xor_sync(0xffffffffu, static_cast<unsigned int>(__bfloat16_as_ushort(odd ? v0 : v1)), 1));
        const uint32_t pair = odd ? (static_cast<uint32_t>(other) | (static_cast<uint32_t>(mine) << 16))
                                  : (static_cast<uint32_t>(mine) | (static_cast<uint32_t>(other) << 16));
        const int tok = i + odd;
        if (tok < nvalid && row_ok)
          *reinterpret_cast<uint32_t*>(ybase + static_cast<size_t>(row_base + tok) * out_ld) = pair;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

template <int BN, int STAGES, int NBUF, bool NCAT>
cudaError_t launch_cfg(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const CUtensorMap& x32,
                       const GemmParams& p, int grid, cudaStream_t stream) {
  using C = Cfg<BN, STAGES, NBUF, NCAT>;
  static bool attr[64] = {false};
  int dev = 0;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return de;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(grouped_gemm_kernel<BN, STAGES, NBUF, NCAT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  grouped_gemm_kernel<BN, STAGES, NBUF, NCAT><<<grid, NUM_THREADS, C::SMEM_BYTES, stream>>>(w0, w1, x, x32, p);
  return cudaGetLastError();
}

}  // namespace gg

// Token tile for a launch over `tokens` tokens: no group can hold more than
// `tokens` rows, so small batches get narrow tiles and many TMEM buffers.
int gemm_tile_tokens(int tokens) {
  if (tokens <= 32) return 32;
  if (tokens <= 64) return 64;
  if (tokens <= 128) return 128;
  return 160;
}

cudaError_t launch_grouped_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                                const CUtensorMap& x32, const GemmParams& p, int tile, int grid, cudaStream_t stream) {
  if (p.n_groups > gg::MAX_GROUPS - 1 || (p.n_mat != 1 && p.n_mat != 2))
    return cudaErrorInvalidValue;
  switch (tile) {
    case 32: return gg::launch_cfg<32, 8, 8, true>(w0, w1, x, x32, p, grid, stream);
    case 64: return gg::launch_cfg<64, 6, 4, true>(w0, w1, x, x32, p, grid, stream);
    case 128: return gg::launch_cfg<128, 4, 2, true>(w0, w1, x, x32, p, grid, stream);
    case 160: return gg::launch_cfg<160, 4, 3, false>(w0, w1, x, x32, p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dsmoe
