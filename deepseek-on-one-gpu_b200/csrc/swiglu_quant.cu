// SwiGLU + FP8 hi/lo split of the down-projection input.
//
// For every permuted row r (one (token, expert) pair) the gate/up GEMM left
// [g | u] in bf16. This kernel forms
//     h = bf16( bf16(silu(g)) * u )          (inference/ops.py:190-192: the
//                                             reference's F.silu on bf16 and
//                                             the bf16 product; silu in fp32
//                                             with the fast exp / divide)
// and stores it in the down GEMM's activation format: one fp32 scale per row
// and two e4m3 terms, h ~= (hi + lo) * scale. One warp per row. Rows of up to
// 2048 features are done in one pass: every lane loads all of its g and u
// vectors first (16 loads in flight), and keeps its 64 values of h packed in
// 32 registers (h is exactly representable in bf16) while the warp reduces
// the row amax. Wider rows take two passes (the second re-reads g and u).
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace sq {
// silu(x) = x / (1 + e^-x) in fp32 with the fast exp and divide: a few ulp
// of fp32 from the exactly rounded value, so bf16(silu(x)) can differ from
// the reference's in its last bit for a small fraction of elements (the
// kernel is bound by instruction issue; this halves its instructions).
__device__ __forceinline__ float silu_f32(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// h = bf16(bf16(silu(g)) * u) for 8 consecutive columns as 4 bf16x2 pairs:
// the product of two bf16 values is exact in fp32, so the packed bf16
// multiply rounds it exactly as the reference's bf16 tensor product does.
__device__ __forceinline__ void swiglu8(const uint4& gv, const uint4& uv, __nv_bfloat162* h) {
  const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
  const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 g = __bfloat1622float2(g2[i]);
    h[i] = __hmul2_rn(__floats2bfloat162_rn(silu_f32(g.x), silu_f32(g.y)), u2[i]);
  }
}

__device__ __forceinline__ float amax8(const __nv_bfloat162* h, float amax) {
  __nv_bfloat162 m = __habs2(h[0]);
#pragma unroll
  for (int i = 1; i < 4; ++i) m = __hmax2(m, __habs2(h[i]));
  const float2 f = __bfloat1622float2(m);
  return fmaxf(amax, fmaxf(f.x, f.y));
}

// Split 8 values (already multiplied by 448 / amax) into hi and lo e4m3 terms
// and store them at hi_dst / lo_dst.
__device__ __forceinline__ void split_store8(const float* q, uint8_t* hi_dst, uint8_t* lo_dst) {
  uint32_t hw[2], lw[2];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const uint16_t h2 = f32x2_to_e4m3x2(q[i], q[i + 1]);
    const uint16_t l2 = f32x2_to_e4m3x2(q[i] - e4m3_to_f32(static_cast<uint8_t>(h2 & 0xff)),
                                        q[i + 1] - e4m3_to_f32(static_cast<uint8_t>(h2 >> 8)));
    if ((i & 2) == 0) {
      hw[i >> 2] = h2;
      lw[i >> 2] = l2;
    } else {
      hw[i >> 2] |= static_cast<uint32_t>(h2) << 16;
      lw[i >> 2] |= static_cast<uint32_t>(l2) << 16;
    }
  }
  *reinterpret_cast<uint2*>(hi_dst) = make_uint2(hw[0], hw[1]);
  *reinterpret_cast<uint2*>(lo_dst) = make_uint2(lw[0], lw[1]);
}

constexpr int MAX_GROUPS = 264;

// Group tables of the permuted rows in shared memory: row r is a real
// (token, expert) row if it lies in group g's segment below its count; the
// 32-row padding at each segment's end is skipped (the down GEMM reads it but
// discards the columns).
__device__ __forceinline__ void load_tables(const int32_t* row_start, const int32_t* counts, int n_groups,
                                            int* s_rs, int* s_cnt) {
  for (int i = threadIdx.x; i <= n_groups; i += blockDim.x) {
    s_rs[i] = row_start[i];
    if (i < n_groups) s_cnt[i] = counts[i];
  }
  __syncthreads();
}

__device__ __forceinline__ bool real_row(int row, int n_groups, const int* s_rs, const int* s_cnt) {
  if (row >= s_rs[n_groups]) return false;
  int lo = 0, hi = n_groups;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_rs[mid] <= row) lo = mid; else hi = mid;
  }
  return row - s_rs[lo] < s_cnt[lo];
}

// One pass, F <= 256 * NIT.
template <int NIT>
__global__ void __launch_bounds__(256) swiglu_quant_1pass(const __nv_bfloat16* __restrict__ gu, int F,
                                                          const int32_t* __restrict__ row_start,
                                                          const int32_t* __restrict__ counts, int n_groups, int P,
                                                          uint8_t* __restrict__ hq, float* __restrict__ hs) {
  __shared__ int s_rs[MAX_GROUPS + 1], s_cnt[MAX_GROUPS];
  load_tables(row_start, counts, n_groups, s_rs, s_cnt);
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (!real_row(row, n_groups, s_rs, s_cnt)) return;
  const __nv_bfloat16* g_row = gu + static_cast<size_t>(row) * 2 * F;
  const __nv_bfloat16* u_row = g_row + F;
  uint4 gv[NIT], uv[NIT];
#pragma unroll
  for (int it = 0; it < NIT; ++it) {
    const int col = it * 256 + lane * 8;
    if (col < F) {
      gv[it] = __ldg(reinterpret_cast<const uint4*>(g_row + col));
      uv[it] = __ldg(reinterpret_cast<const uint4*>(u_row + col));
    }
  }
  __nv_bfloat162 hb[NIT * 4];
  float amax = 0.f;
#pragma unroll
  for (int it = 0; it < NIT; ++it) {
    const int col = it * 256 + lane * 8;
    if (col < F) {
      swiglu8(gv[it], uv[it], hb + it * 4);
      amax = amax8(hb + it * 4, amax);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float inv = amax > 0.f ? 448.f / amax : 0.f;
  if (lane == 0) hs[row] = amax / 448.f;
  uint8_t* hi_row = hq + static_cast<size_t>(row) * F;
  uint8_t* lo_row = hq + (static_cast<size_t>(P) + row) * F;
#pragma unroll
  for (int it = 0; it < NIT; ++it) {
    const int col = it * 256 + lane * 8;
    if (col < F) {
      float q[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 v = __bfloat1622float2(hb[it * 4 + i]);
        q[2 * i] = v.x * inv;
        q[2 * i + 1] = v.y * inv;
      }
      split_store8(q, hi_row + col, lo_row + col);
    }
  }
}

__global__ void __launch_bounds__(256) swiglu_quant_kernel(const __nv_bfloat16* __restrict__ gu, int F,
                                                           const int32_t* __restrict__ row_start,
                                                           const int32_t* __restrict__ counts, int n_groups, int P,
                                                           uint8_t* __restrict__ hq, float* __restrict__ hs) {
  __shared__ int s_rs[MAX_GROUPS + 1], s_cnt[MAX_GROUPS];
  load_tables(row_start, counts, n_groups, s_rs, s_cnt);
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (!real_row(row, n_groups, s_rs, s_cnt)) return;
  const __nv_bfloat16* g_row = gu + static_cast<size_t>(row) * 2 * F;
  const __nv_bfloat16* u_row = g_row + F;
  uint8_t* hi_row = hq + static_cast<size_t>(row) * F;
  uint8_t* lo_row = hq + (static_cast<size_t>(P) + row) * F;
  float amax = 0.f;
  for (int col = lane * 8; col < F; col += 256) {
    __nv_bfloat162 h[4];
    swiglu8(__ldg(reinterpret_cast<const uint4*>(g_row + col)), __ldg(reinterpret_cast<const uint4*>(u_row + col)), h);
    amax = amax8(h, amax);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float inv = amax > 0.f ? 448.f / amax : 0.f;
  if (lane == 0) hs[row] = amax / 448.f;
  for (int col = lane * 8; col < F; col += 256) {
    __nv_bfloat162 h[4];
    swiglu8(__ldg(reinterpret_cast<const uint4*>(g_row + col)), __ldg(reinterpret_cast<const uint4*>(u_row + col)), h);
    float q[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 v = __bfloat1622float2(h[i]);
      q[2 * i] = v.x * inv;
      q[2 * i + 1] = v.y * inv;
    }
    split_store8(q, hi_row + col, lo_row + col);
  }
}
}  // namespace sq

cudaError_t launch_swiglu_quant(const __nv_bfloat16* gu, int F, const int32_t* row_start, const int32_t* counts,
                                int n_groups, int P, uint8_t* hq, float* hs, cudaStream_t stream) {
  if (P == 0) return cudaSuccess;
  if (n_groups < 1 || n_groups > sq::MAX_GROUPS) return cudaErrorInvalidValue;
  const int blocks = (P * 32 + 255) / 256;
  if (F <= 2048)
    sq::swiglu_quant_1pass<8><<<blocks, 256, 0, stream>>>(gu, F, row_start, counts, n_groups, P, hq, hs);
  else
    sq::swiglu_quant_kernel<<<blocks, 256, 0, stream>>>(gu, F, row_start, counts, n_groups, P, hq, hs);
  return cudaGetLastError();
}

}  // namespace dsmoe
