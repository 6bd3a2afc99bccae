// K5: weighted combine / un-permute with the shared expert.
//
// For token t, with y the down-projection rows (bf16, one per (token, k)
// pair and one shared-expert row per token):
//   acc = 0 (bf16)
//   for k in 0..top_k-1:  acc = bf16(acc + bf16(bf16(w[t,k]) * y[pos[t,k]]))
//   out[t] = bf16(y_shared[t] + bf16(acc * scale))
// Without a shared expert (a rank's share of an expert-parallel step) the
// output is bf16(acc): the rank's partial, summed and scaled by the caller.
// With a residual r (the MoE layer's FFN half, inference/forward.py:109) the
// output is bf16(r[t] + out[t]): the layer's `hidden + ffn_out` in bf16.
// With peer outputs (expert parallelism over peer memory) row t is written to
// the return buffer of the rank it came from, origin[t] = (rank, k), at row
// me * cap + k of that rank's buffer (peer_out[rank] in this process's
// address space).
// This is the reference's arithmetic (inference/forward.py:137,151,153): the
// fp32 0-dim weight times a bf16 row yields bf16 (the weight is rounded to
// bf16 by type promotion), the running sum is bf16 and accumulates in top-k
// order, and the final ``shared + routed * routed_scaling_factor`` is bf16.
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace cb {
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ y, int T, int H,
                                                      const int32_t* __restrict__ pos,
                                                      const float* __restrict__ w, int top_k,
                                                      const int32_t* __restrict__ row_start, float scale,
                                                      int has_shared, const __nv_bfloat16* __restrict__ residual,
                                                      __nv_bfloat16* __restrict__ out,
                                                      const int32_t* __restrict__ origin,
                                                      const uint64_t* __restrict__ peer_out, int me, int cap,
                                                      const int32_t* __restrict__ n_rows) {
  // Rows beyond the device-side count are skipped. A CTA handles rows
  // blockIdx.x, blockIdx.x + gridDim.x, ...: one row per CTA when the output
  // is local, a persistent grid when rows go to other GPUs, so that the one
  // system-scope fence that makes them visible there is paid per CTA rather
  // than per row.
  const int rows = n_rows ? min(T, *n_rows) : T;
  __shared__ int s_row[8];
  __shared__ __nv_bfloat162 s_w2[8];  // bf16(w[t,k]) in both halves
  for (int t = blockIdx.x; t < rows; t += gridDim.x) {
    __syncthreads();  // the previous row's s_row / s_w2 are no longer read
    if (threadIdx.x < top_k) {
      s_row[threadIdx.x] = pos[static_cast<size_t>(t) * top_k + threadIdx.x];
      const __nv_bfloat16 wb = __float2bfloat16_rn(w[static_cast<size_t>(t) * top_k + threadIdx.x]);
      s_w2[threadIdx.x] = __halves2bfloat162(wb, wb);
    }
    __syncthreads();
    const int srow = row_start[0] + t;
    const int nchunks = H / 8;
    __nv_bfloat16* orow = out + static_cast<size_t>(t) * H;
    if (peer_out) {
      const int src_rank = origin[2 * t], k = origin[2 * t + 1];
      orow = reinterpret_cast<__nv_bfloat16*>(peer_out[src_rank]) + (static_cast<size_t>(me) * cap + k) * H;
    }
    for (int c = threadIdx.x; c < nchunks; c += blockDim.x) {
      // All rows of the token are loaded before the ordered bf16 sum so that
      // the loads overlap.
      uint4 v[8];
  #pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = k < top_k ? s_row[k] : -1;
        v[k] = r >= 0 ? __ldg(reinterpret_cast<const uint4*>(y + static_cast<size_t>(r) * H) + c) : make_uint4(0, 0, 0, 0);
      }
      const uint4 sv = has_shared ? __ldg(reinterpret_cast<const uint4*>(y + static_cast<size_t>(srow) * H) + c)
                                  : make_uint4(0, 0, 0, 0);
      // Packed bf16x2 arithmetic: each multiply and each add rounds its exact
      // result to bf16 once, which is what the reference's bf16 tensor ops do
      // (they compute in fp32, exact for a product of two bf16 values and
      // innocuously double-rounded for a sum, then round to bf16). The _rn
      // forms keep the compiler from fusing a multiply and the following add
      // into one FMA, which would skip the product's rounding.
      __nv_bfloat162 acc[4];
  #pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = __float2bfloat162_rn(0.f);
  #pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k >= top_k || s_row[k] < 0) continue;
        const __nv_bfloat162* vb = reinterpret_cast<const __nv_bfloat162*>(&v[k]);
        const __nv_bfloat162 wk = s_w2[k];
  #pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = __hadd2_rn(acc[i], __hmul2_rn(wk, vb[i]));
      }
      uint4 o;
      __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
      if (has_shared) {
        // shared + bf16(routed * scale): the scale stays fp32 (a Python float
        // in the reference), so this product is taken in fp32 and rounded
        const __nv_bfloat162* sb = reinterpret_cast<const __nv_bfloat162*>(&sv);
  #pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a = __bfloat1622float2(acc[i]);
          ob[i] = __hadd2_rn(sb[i], __floats2bfloat162_rn(a.x * scale, a.y * scale));
        }
      } else {
  #pragma unroll
        for (int i = 0; i < 4; ++i) ob[i] = acc[i];
      }
      if (residual) {
        const uint4 rv = __ldg(reinterpret_cast<const uint4*>(residual + static_cast<size_t>(t) * H) + c);
        const __nv_bfloat162* rb = reinterpret_cast<const __nv_bfloat162*>(&rv);
  #pragma unroll
        for (int i = 0; i < 4; ++i) ob[i] = __hadd2_rn(rb[i], ob[i]);
      }
      reinterpret_cast<uint4*>(orow)[c] = o;
    }
  }
  if (peer_out) __threadfence_system();
}
}  // namespace cb

cudaError_t launch_combine(const __nv_bfloat16* y, int T, int H, const int32_t* pos, const float* w, int top_k,
                           const int32_t* row_start, float scale, int has_shared, const __nv_bfloat16* residual,
                           __nv_bfloat16* out, cudaStream_t stream, const int32_t* origin, const uint64_t* peer_out,
                           int me, int cap, const int32_t* n_rows) {
  if (T == 0) return cudaSuccess;
  int grid = T;
  if (peer_out) {
    static int n_sm[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (n_sm[dev] == 0 && cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return cudaErrorInvalidDevice;
    grid = T < 4 * n_sm[dev] ? T : 4 * n_sm[dev];
  }
  cb::combine_kernel<<<grid, 256, 0, stream>>>(y, T, H, pos, w, top_k, row_start, scale, has_shared, residual, out,
                                            origin, peer_out, me, cap, n_rows);

  return cudaGetLastError();
}

}  // namespace dsmoe
