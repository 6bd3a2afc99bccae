// RMSNorm in front of the MoE block (inference/ops.py:10-13, applied at
// inference/forward.py:97):
//     r = 1 / sqrt(mean_j(x_j^2) + eps)            fp32
//     y = bf16( bf16(x * r) * w )                  x, w, y bf16
// The reference computes x.float() * r, rounds to x's dtype, then multiplies
// by the bf16 weight (a bf16 product, rounded once). Here the mean is a
// per-thread fp32 sum then a tree over the block, so it may differ from
// torch's CPU reduction in the last bit of r; 1/sqrt uses the correctly
// rounded sqrtf and division, like torch's CPU rsqrt.
//
// One CTA of 128 threads per row; rows of up to 128 * 8 * MAXC elements keep
// their values in registers between the sum and the scaling (one HBM read and
// one write per element).
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace rn {
constexpr int THREADS = 128;
constexpr int MAXC = 8;  // 16-byte chunks per thread held in registers: H <= 8192

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) t += red[i];  // fixed order: every thread gets the same value
  return t;
}

__device__ __forceinline__ uint4 scale8(uint4 xv, uint4 wv, float r) {
  const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
  const __nv_bfloat16* wb = reinterpret_cast<const __nv_bfloat16*>(&wv);
  uint4 o;
  __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    ob[i] = __float2bfloat16_rn(bf16_round(__bfloat162float(xb[i]) * r) * __bfloat162float(wb[i]));
  return o;
}

__global__ void __launch_bounds__(THREADS) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w, float eps, int H,
                                                          __nv_bfloat16* __restrict__ y) {
  __shared__ float red[THREADS / 32];
  const size_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * H);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * H);
  const int nchunks = H / 8;
  if (nchunks <= THREADS * MAXC) {
    uint4 v[MAXC];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * THREADS;
      if (c < nchunks) {
        v[i] = __ldg(xr + c);
        const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float f = __bfloat162float(b[k]);
          ss = fmaf(f, f, ss);
        }
      }
    }
    const float r = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(H) + eps);
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = threadIdx.x + i * THREADS;
      if (c < nchunks) yr[c] = scale8(v[i], __ldg(wr + c), r);
    }
  } else {
    float ss = 0.f;
    for (int c = threadIdx.x; c < nchunks; c += THREADS) {
      const uint4 v = __ldg(xr + c);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float f = __bfloat162float(b[k]);
        ss = fmaf(f, f, ss);
      }
    }
    const float r = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(H) + eps);
    for (int c = threadIdx.x; c < nchunks; c += THREADS) yr[c] = scale8(__ldg(xr + c), __ldg(wr + c), r);
  }
}
}  // namespace rn

cudaError_t launch_rmsnorm(const void* x, const void* w, float eps, int T, int H, void* y, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  rn::rmsnorm_kernel<<<T, rn::THREADS, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                    static_cast<const __nv_bfloat16*>(w), eps, H,
                                                    static_cast<__nv_bfloat16*>(y));
  return cudaGetLastError();
}

}  // namespace dsmoe
