// K1a: router logits on tcgen05 (bf16 x bf16 -> fp32), split over K.
//
//   partial[ks][t][e] = sum_{k in split ks} x[t, k] * Wg[e, k]
//
// (inference/ops.py:224 computes hidden.float() @ gate_weight.float().T; bf16
// products are exact in fp32, so only the order of the fp32 additions differs.)
// The selection kernel (router.cu) adds the ksplit partials in a fixed order,
// so the logits are deterministic run to run.
//
// One CTA per (128-token tile, K split): the token tile is the 128-row A
// operand, all experts (up to 256) are the N operand, K advances 64 elements
// (128 bytes) per stage. Warp 0 issues TMA, warp 1 allocates TMEM and issues
// the MMAs, warps 2-5 read the 128 x E accumulator back and store it.
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace rtc {
constexpr int BM = 128;      // tokens per tile
constexpr int BKE = 64;      // K elements per stage (128 bytes of bf16)
constexpr int MAX_E = 256;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * 128;
constexpr int B_BYTES = MAX_E * 128;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int BAR_OFF = STAGES * STAGE_BYTES;
constexpr int MISC_OFF = BAR_OFF + 8 * (2 * STAGES + 1);
constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
constexpr int NUM_THREADS = 6 * 32;

__global__ void __launch_bounds__(NUM_THREADS, 1)
router_logits_tc(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_g, float* partial,
                 int T, int E, int ksteps_per_split, int ksteps_total, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + MISC_OFF + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * BM;
  const int ks = blockIdx.y;
  const int kbeg = ks * ksteps_per_split;
  const int kend = min(ksteps_total, kbeg + ksteps_per_split);
  const int nk = kend - kbeg;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_g);
  }
  if (warp == 1) tmem_alloc(s_tmem, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_x = policy_evict_first();
      const uint64_t pol_g = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int k = 0; k < nk; ++k) {
        if (!mbar_wait(&empty[stage], phase ^ 1, status, kDevTimeoutProducer, s_abort)) break;
        uint8_t* st = smem + stage * STAGE_BYTES;
        mbar_arrive_expect_tx(&full[stage], A_BYTES + E * 128);
        tma_load_2d(st, &tm_x, &full[stage], (kbeg + k) * BKE, t0, pol_x);
        tma_load_2d(st + A_BYTES, &tm_g, &full[stage], (kbeg + k) * BKE, 0, pol_g);
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      const int n_drain = issued < STAGES ? issued : STAGES;
      for (int i = 0; i < n_drain; ++i) {
        if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
        mbar_wait_settle(&full[stage], phase, status, kDevTimeoutProducer);  // copies in flight land
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(BM, E);
      int stage = 0;
      uint32_t phase = 0;
      for (int k = 0; k < nk; ++k) {
        if (!mbar_wait(&full[stage], phase, status, kDevTimeoutMma, s_abort)) break;
        tc_fence_after();
        const uint32_t sbase = smem_u32(smem + stage * STAGE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKE / 16; ++kk)
          mma_bf16(tmem, umma_desc_sw128(sbase + kk * 32), umma_desc_sw128(sbase + A_BYTES + kk * 32), idesc,
                   (k | kk) != 0);
        mma_commit(&empty[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      mma_commit(done);
      // the MMAs finish with TMEM before it is freed, also after an abort
      mbar_wait_settle(done, 0, status, kDevTimeoutMma);
    }
  } else {
    // epilogue: warp w owns TMEM lanes 32*(w%4) .. +31 = tokens of the tile
    const int quad = warp & 3;
    const bool ok = mbar_wait(done, 0, status, kDevTimeoutEpilogue, s_abort);
    tc_fence_after();
    const int t = t0 + quad * 32 + lane;
    float* out = partial + (static_cast<size_t>(ks) * T + t) * E;
    for (int c = 0; c < E; c += 32) {
      float v[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + c, v);
      tmem_ld_wait();
      if (ok && t < T) {
        const float m = nk > 0 ? 1.f : 0.f;  // an empty split contributes zeros
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(out + c + i) = make_float4(m * v[i], m * v[i + 1], m * v[i + 2], m * v[i + 3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 256);
}
}  // namespace rtc

// K splits for T tokens: enough CTAs to cover the SMs, at least 4 K steps per
// split, and no empty split (the selection kernel adds exactly this many).
int router_tc_ksplit(int T, int H, int num_sms) {
  const int tiles = (T + rtc::BM - 1) / rtc::BM;
  const int ksteps = H / rtc::BKE;
  int ks = (num_sms + tiles - 1) / tiles;
  if (ks > 16) ks = 16;
  if (ks > ksteps / 4) ks = ksteps / 4;
  if (ks < 1) ks = 1;
  const int per = (ksteps + ks - 1) / ks;
  return (ksteps + per - 1) / per;
}

cudaError_t launch_router_logits_tc(const CUtensorMap& tm_x, const CUtensorMap& tm_g, float* partial, int T, int H,
                                    int E, int ksplit, int* status, cudaStream_t stream) {
  if (E > rtc::MAX_E || E % 16 || H % rtc::BKE) return cudaErrorInvalidValue;
  static bool attr[64] = {false};
  int dev = 0;
  const cudaError_t de = cudaGetDevice(&dev);
  if (de != cudaSuccess) return de;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(rtc::router_logits_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, rtc::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  const int ksteps = H / rtc::BKE;
  const int per = (ksteps + ksplit - 1) / ksplit;
  dim3 grid((T + rtc::BM - 1) / rtc::BM, ksplit);
  rtc::router_logits_tc<<<grid, rtc::NUM_THREADS, rtc::SMEM_BYTES, stream>>>(tm_x, tm_g, partial, T, E, per, ksteps,
                                                                              status);
  return cudaGetLastError();
}

}  // namespace dsmoe
