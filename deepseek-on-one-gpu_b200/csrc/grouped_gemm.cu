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
// Warp roles (one CTA per SM, persistent over work units):
//   warp 0      TMA producer (one thread)
//   warp 1      TMEM allocator + MMA issuer for even K steps (one thread)
//   warp 2      MMA issuer for odd K steps (one thread)
//   warp 3      unit planner: decodes the CTA's work units ahead of time into
//               a shared-memory ring (rows, weight row, MMA width and the
//               unit's first 32 weight scales), so that no other role waits on
//               a chain of dependent global loads at a unit boundary
//   warps 4..   epilogue, 16 warps: warp w reads TMEM lane quadrant (w % 4)
//               and one column group of BN / 4 columns; a K step's partial
//               (40 columns at BN 160) is read with all its TMEM loads in
//               flight together and one wait.
// Two issuers: a thread that waits on an mbarrier between its MMA batches
// leaves the tensor pipe idle for a few hundred cycles each time; with the
// K steps split by parity one issuer's MMAs run while the other waits. Every
// K step writes its own TMEM buffer and smem stage, so the two streams are
// independent; each issuer commits only its own MMAs.
// At a unit boundary the epilogue warps store the finished tile and start the
// next one from values already in shared memory; the MMA meanwhile runs up to
// NBUF - 1 K steps of the next unit ahead.
// Activation tiles are one TMA box of BN rows per term (hi, lo); groups of at
// most 64 tokens use 32-row boxes instead so decode steps do not pull BN rows.
// Work unit = (group, 128-feature tile, BN-token tile); units are ordered
// group-major, then feature tile, then token tile; CTA b takes units b,
// b + gridDim.x, ...
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace gg {
constexpr int BM = 128;   // weight rows (output features) per tile
constexpr int BK = 128;   // K bytes per stage
constexpr int SUB = 32;   // token rows per small activation TMA box
constexpr int MAX_GROUPS = 264;
constexpr int RING = 4;       // unit-plan entries in flight
constexpr int SW_WIN = 32;    // weight scales per window (one per lane)
constexpr int PLAN_WARP = 3;
constexpr int EPI_WARP0 = 4;

// One work unit as the planner hands it to the other roles.
struct UnitPlan {
  int32_t ncols;    // valid token columns of the tile
  int32_t row0;     // first activation / output row of the tile
  int32_t wrow;     // first weight row in the bank map (slot * M + feature tile * 128)
  int32_t mat;      // weight matrix (0 or 1)
  int32_t mrow;     // first output feature inside the matrix
  int32_t nmma;     // MMA N (columns written to TMEM per K step)
  int32_t wsc_off;  // offset of the tile's weight-scale row ([K/128] floats)
  int32_t pad;
  float sw[SW_WIN]; // weight scales of K blocks 0..31
};
static_assert(sizeof(UnitPlan) == 160, "plan entry size");

template <int BN_, int STAGES_, int NBUF_, bool NCAT_, int EPI_WARPS_>
struct Cfg {
  static constexpr int BN = BN_;                  // max tokens per tile
  static constexpr int STAGES = STAGES_;
  static constexpr int NBUF = NBUF_;              // TMEM accumulator buffers (MMA runs NBUF-1 K steps ahead)
  // hi and lo rows are adjacent in shared memory; for tiles of up to 128
  // tokens one MMA covers both (N = 2 * BN, columns [0,BN) hi, [BN,2BN) lo),
  // halving the MMA count; wider tiles accumulate hi then lo along K.
  static constexpr bool NCAT = NCAT_;
  static constexpr int EPI_WARPS = EPI_WARPS_;
  static constexpr int NUM_CG = EPI_WARPS / 4;    // column groups
  static constexpr int NUM_THREADS = (EPI_WARP0 + EPI_WARPS) * 32;
  static constexpr int TCOLS = NCAT ? 2 * BN : BN;  // TMEM columns per buffer
  static constexpr int EPI_COLS = BN / NUM_CG;    // accumulator columns per epilogue warp
  // columns per TMEM load: the warp's whole slice where the partial is one
  // term, 16-column pieces of hi and lo where it is two
  static constexpr int CHUNK = NCAT ? (EPI_COLS < 16 ? EPI_COLS : 16) : EPI_COLS;
  static constexpr int XH_OFF = BM * BK;
  static constexpr int XL_OFF = XH_OFF + BN * BK;
  static constexpr int STAGE_BYTES = XL_OFF + BN * BK;  // multiple of 1024 for BN % 8 == 0
  static constexpr int TMEM_COLS = NBUF * TCOLS <= 32 ? 32 : NBUF * TCOLS <= 64 ? 64 : NBUF * TCOLS <= 128 ? 128
                                   : NBUF * TCOLS <= 256 ? 256 : 512;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  // barriers: full[S], empty[S], tfull[NBUF], tempty[NBUF], done, ufull[RING], uempty[RING]
  static constexpr int NUM_BARS = 2 * STAGES + 2 * NBUF + 1 + 2 * RING;
  static constexpr int MISC_OFF = BAR_OFF + 8 * NUM_BARS;
  static constexpr int PLAN_OFF = ((MISC_OFF + 16 + 15) / 16) * 16;
  static constexpr int SMEM_BYTES = PLAN_OFF + RING * static_cast<int>(sizeof(UnitPlan)) + 1024;  // + alignment slack
  static_assert(EPI_WARPS % 4 == 0 && BN % NUM_CG == 0, "epilogue split");
  static_assert(EPI_COLS <= 40 && (CHUNK == 8 || CHUNK == 16 || CHUNK == 32 || CHUNK == 40) &&
                    EPI_COLS % CHUNK == 0, "epilogue columns");
  static_assert(BN % 32 == 0 && BN <= 256 && NBUF * TCOLS <= 512 && (!NCAT || 2 * BN <= 256), "tile shape");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// unit -> (group, feature tile, token tile), from the unit prefix sums
template <int BN>
__device__ __forceinline__ void decode_unit(int u, int n_groups, const int* __restrict__ ustart,
                                            const int* __restrict__ counts, int& g, int& mt, int& nt) {
  int lo = 0, hi = n_groups;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(ustart + mid) <= u) lo = mid; else hi = mid;
  }
  g = lo;
  const int ntiles = (__ldg(counts + g) + BN - 1) / BN;
  const int local = u - __ldg(ustart + g);
  mt = local / ntiles;
  nt = local - mt * ntiles;
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v) {
  if constexpr (N == 40) {
    tmem_ld32(taddr, v);
    tmem_ld8(taddr + 32, v + 32);
  } else if constexpr (N == 32) tmem_ld32(taddr, v);
  else if constexpr (N == 16) tmem_ld16(taddr, v);
  else tmem_ld8(taddr, v);
}

template <int BN_, int STAGES_, int NBUF_, bool NCAT_, int EPI_WARPS_>
__global__ void __launch_bounds__(Cfg<BN_, STAGES_, NBUF_, NCAT_, EPI_WARPS_>::NUM_THREADS, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                    const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_x32,
                    const GemmParams p) {
  using C = Cfg<BN_, STAGES_, NBUF_, NCAT_, EPI_WARPS_>;
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
  uint64_t* ufull = done_bar + 1;
  uint64_t* uempty = ufull + RING;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);
  UnitPlan* plan = reinterpret_cast<UnitPlan*>(smem + C::PLAN_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NG = p.n_groups;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], C::EPI_WARPS);
    }
    mbar_init(done_bar, 2);
    for (int r = 0; r < RING; ++r) {
      mbar_init(&ufull[r], 32);                    // every lane of the planner warp
      mbar_init(&uempty[r], 3 + C::EPI_WARPS);     // producer, two issuers, epilogue warps
    }
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
  const int total_units = __ldg(p.unit_start + NG);
  const int n_kb = p.K / BK;
  // 128-row tiles per matrix; a ragged last tile (single-slot linear layers
  // such as 576 outputs) reads zero-filled rows past the end of the weight
  // and stores only rows < M.
  const int mt_per_mat = (p.M + BM - 1) / BM;

  if (warp == PLAN_WARP) {
    // ------------------------------------------------------------- planner
    int i = 0;
    for (int u = blockIdx.x; u < total_units; u += gridDim.x, ++i) {
      int g, mt, nt;
      decode_unit<BN>(u, NG, p.unit_start, p.counts, g, mt, nt);
      const int slot = __ldg(p.slot_of + g);
      if (slot < 0 || slot >= p.n_slots) {
        if (lane == 0) atomicCAS(p.status, 0, kDevBadSlot);
        *s_abort = 1;  // every role leaves its next wait
        break;
      }
      const int mat = mt >= mt_per_mat;
      const int mtl = mt - mat * mt_per_mat;
      const int wsc_off = (slot * mt_per_mat + mtl) * n_kb;
      const float swv = lane < n_kb ? __ldg((mat ? p.wscale1 : p.wscale0) + wsc_off + lane) : 0.f;
      const int ncols = min(BN, __ldg(p.counts + g) - nt * BN);
      const int row0 = __ldg(p.row_start + g) + nt * BN;
      const int ri = i % RING;
      if (!mbar_wait(&uempty[ri], ((i / RING) & 1) ^ 1, p.status, kDevTimeoutProducer, s_abort)) break;
      UnitPlan* e = plan + ri;
      if (lane == 0) {
        e->ncols = ncols;
        e->row0 = row0;
        e->wrow = slot * p.M + mtl * BM;
        e->mat = mat;
        e->mrow = mtl * BM;
        e->nmma = C::NCAT ? 2 * BN : (ncols + 15) & ~15;
        e->wsc_off = wsc_off;
      }
      e->sw[lane] = swv;
      mbar_arrive(&ufull[ri]);  // each lane publishes its own writes
    }
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      int i = 0;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++i) {
        const int ri = i % RING;
        if (!mbar_wait(&ufull[ri], (i / RING) & 1, p.status, kDevTimeoutProducer, s_abort)) break;
        const UnitPlan* e = plan + ri;
        const int ncols = e->ncols, row0 = e->row0, wrow = e->wrow, mat = e->mat;
        mbar_arrive(&uempty[ri]);
        const CUtensorMap* tw = mat ? &tm_w1 : &tm_w0;
        const int nsub = (ncols + SUB - 1) / SUB;
        // A few 32-row boxes beat one big box; four or more cost more than the
        // rows they save (a 128-token tile as 4 boxes: +8% kernel time).
        const bool small = BN == SUB || (nsub * SUB < BN && nsub <= 2);
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
      // the CTA may exit (normally they were consumed already; after an
      // abort they may still be in flight).
      const int n_drain = issued < STAGES ? issued : STAGES;
      for (int d = 0; d < n_drain; ++d) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        mbar_wait_settle(&full[stage], phase, p.status, kDevTimeoutProducer);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ----------------------------------------------------------------- MMA
    if (lane == 0) {
      const int me = warp - 1;  // issues the K steps of this parity
      int step = 0;
      int stage = 0;
      uint32_t phase = 0;
      int tb = 0;
      uint32_t tphase = 0;
      bool ok = true;
      int i = 0;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++i) {
        const int ri = i % RING;
        if (!mbar_wait(&ufull[ri], (i / RING) & 1, p.status, kDevTimeoutMma, s_abort)) break;
        const int N = plan[ri].nmma;
        mbar_arrive(&uempty[ri]);
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
      // barrier's first phase needs one commit from each), also after an abort.
      mma_commit(done_bar);
      mbar_wait_settle(done_bar, 0, p.status, kDevTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // a warp reads the TMEM lanes of quadrant warp % 4
    const int cg = (warp - EPI_WARP0) >> 2;
    const int c0 = cg * EPI_COLS;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int out_ld = p.n_mat * p.M;
    int tb = 0;
    uint32_t tphase = 0;
    bool ok = true;
    int i = 0;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x, ++i) {
      const int ri = i % RING;
      if (!mbar_wait(&ufull[ri], (i / RING) & 1, p.status, kDevTimeoutEpilogue, s_abort)) break;
      const UnitPlan* e = plan + ri;
      const int ncols = e->ncols, row0 = e->row0, mat = e->mat, mrow = e->mrow, wsc_off = e->wsc_off;
      // Weight block scales, one per K block, in 32-block windows: lane i
      // holds kb = 32w + i of window w in register w % 2; window 0 comes from
      // the plan, entering window w refills the other register with window
      // w + 1 from global memory, 32 K steps before it is needed.
      float swr0 = e->sw[lane];
      __syncwarp();
      if (lane == 0) mbar_arrive(&uempty[ri]);
      const float* wsc = (mat ? p.wscale1 : p.wscale0) + wsc_off;
      float swr1 = 32 + lane < n_kb ? __ldg(wsc + 32 + lane) : 0.f;
      const int nvalid = max(0, min(EPI_COLS, ncols - c0));  // valid columns of this warp
      // Per-row activation scales of this warp's columns `lane` and
      // `32 + lane`, loaded now so that the latency hides behind the K loop.
      const int row_base = row0 + c0;
      const float sxv = lane < nvalid ? __ldg(p.sx + row_base + lane) : 0.f;
      const float sxw = 32 + lane < nvalid ? __ldg(p.sx + row_base + 32 + lane) : 0.f;
      float acc[EPI_COLS];
#pragma unroll
      for (int c = 0; c < EPI_COLS; ++c) acc[c] = 0.f;

      for (int kb = 0; kb < n_kb; ++kb) {
        if (!mbar_wait(&tfull[tb], tphase, p.status, kDevTimeoutEpilogue, s_abort)) { ok = false; break; }
        tc_fence_after();
        if ((kb & 31) == 0 && kb >= 32) {
          const int nk = kb + 32 + lane;
          const float v = nk < n_kb ? __ldg(wsc + nk) : 0.f;
          if ((kb >> 5) & 1) swr0 = v; else swr1 = v;
        }
        const float sw = __shfl_sync(0xffffffffu, ((kb >> 5) & 1) ? swr1 : swr0, kb & 31);
#pragma unroll
        for (int q = 0; q < EPI_COLS / CHUNK; ++q) {
          if (q * CHUNK < nvalid) {  // warp-uniform
            const uint32_t ta = tmem_base + lane_base + tb * C::TCOLS + c0 + q * CHUNK;
            float part[CHUNK];
            tmem_ld<CHUNK>(ta, part);
            if constexpr (C::NCAT) {
              float lo[CHUNK];
              tmem_ld<CHUNK>(ta + BN, lo);
              tmem_ld_wait();
#pragma unroll
              for (int c = 0; c < CHUNK; ++c) part[c] += lo[c];
            } else {
              tmem_ld_wait();
            }
            // Packed fp32x2 FMAs: half the issue slots of scalar fmaf, same
            // rounding.
#pragma unroll
            for (int c = 0; c < CHUNK; c += 2)
              fma2(acc[q * CHUNK + c], acc[q * CHUNK + c + 1], part[c], part[c + 1], sw);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[tb]);
        if (++tb == NBUF) { tb = 0; tphase ^= 1; }
      }
      if (!ok) break;
      // Stores of bf16 pairs: for tokens c and c+1, an even lane writes
      // features (lane, lane+1) of token c and its odd neighbour features
      // (lane-1, lane) of token c+1; one shuffle exchanges the halves.
      const int odd = lane & 1;
      const int row_in_mat = mrow + quad * 32 + (lane & ~1);  // the pair's first row
      const bool row_ok = row_in_mat < p.M;  // M is even: the pair is inside or outside together
      __nv_bfloat16* ybase = p.y + mat * p.M + row_in_mat;
#pragma unroll
      for (int c = 0; c < EPI_COLS; c += 2) {
        const float s0 = __shfl_sync(0xffffffffu, c < 32 ? sxv : sxw, c & 31);
        const float s1 = __shfl_sync(0xffffffffu, c + 1 < 32 ? sxv : sxw, (c + 1) & 31);
        const __nv_bfloat16 v0 = __float2bfloat16_rn(acc[c] * s0);
        const __nv_bfloat16 v1 = __float2bfloat16_rn(acc[c + 1] * s1);
        const unsigned short mine = __bfloat16_as_ushort(odd ? v1 : v0);
        const unsigned short other = static_cast<unsigned short>(
            __shfl_xor_sync(0xffffffffu, static_cast<unsigned int>(__bfloat16_as_ushort(odd ? v0 : v1)), 1));
        const uint32_t pair = odd ? (static_cast<uint32_t>(other) | (static_cast<uint32_t>(mine) << 16))
                                  : (static_cast<uint32_t>(mine) | (static_cast<uint32_t>(other) << 16));
        const int tok = c + odd;
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

template <int BN, int STAGES, int NBUF, bool NCAT, int EPI_WARPS>
cudaError_t launch_cfg(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x, const CUtensorMap& x32,
                       const GemmParams& p, int grid, cudaStream_t stream) {
  using C = Cfg<BN, STAGES, NBUF, NCAT, EPI_WARPS>;
  static bool attr[64] = {false};
  int dev = 0;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return de;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(grouped_gemm_kernel<BN, STAGES, NBUF, NCAT, EPI_WARPS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  grouped_gemm_kernel<BN, STAGES, NBUF, NCAT, EPI_WARPS>
      <<<grid, C::NUM_THREADS, C::SMEM_BYTES, stream>>>(w0, w1, x, x32, p);
  return cudaGetLastError();
}

}  // namespace gg

// Token tile for a launch over `tokens` tokens. What matters is the routed
// experts' share, about tokens * top_k / experts rows each (the shared
// expert's tokens rows are split into as many tiles as needed): narrow tiles
// keep a unit's MMAs as wide as its rows and leave room for more stages and
// TMEM buffers. Measured on the MoE block (256+1 experts, one B200, ms per
// step for tiles of 32 / 64 / 160 tokens): T=128 1.81 / 2.21 / 2.73 (128),
// T=256 1.99 / 2.51 / 2.65, T=512 2.06 / 2.51 / 2.44, T=1024 3.23 / 2.52 /
// 2.88, T=2048 5.43 / 4.14 / 3.54.
int gemm_tile_tokens(int tokens) {
  if (tokens <= 512) return 32;
  if (tokens <= 1024) return 64;
  return 160;
}

cudaError_t launch_grouped_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                                const CUtensorMap& x32, const GemmParams& p, int tile, int grid, cudaStream_t stream) {
  if (p.n_groups > gg::MAX_GROUPS - 1 || (p.n_mat != 1 && p.n_mat != 2))
    return cudaErrorInvalidValue;
  switch (tile) {
    case 32: return gg::launch_cfg<32, 8, 8, true, 16>(w0, w1, x, x32, p, grid, stream);
    case 64: return gg::launch_cfg<64, 6, 4, true, 16>(w0, w1, x, x32, p, grid, stream);
    case 128: return gg::launch_cfg<128, 4, 2, true, 16>(w0, w1, x, x32, p, grid, stream);
    case 160: return gg::launch_cfg<160, 4, 3, false, 16>(w0, w1, x, x32, p, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dsmoe
