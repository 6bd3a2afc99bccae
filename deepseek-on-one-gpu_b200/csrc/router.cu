// K1: router — fp32 logits, sigmoid scores, group-limited top-k selection.
//
// Reference semantics (mode 0), inference/ops.py:209-257:
//   logits = x.float() @ Wg.float().T                   (:224)
//   s = sigmoid(logits)                                  (:225)
//   group score = max of the group's scores              (:239)
//   keep the topk_group best groups, others -> 0.0       (:240-248)
//   top_k experts by masked score, descending            (:251)
//   w = v / (sum(v) + 1e-9)  if norm_topk_prob           (:254-255)
// Bias-corrected semantics (mode 1, DeepSeek-V3): selection key s + bias,
// group score = sum of the two largest keys, masked groups -> -inf, weights =
// unbiased s at the chosen experts / their sum * routed_scaling_factor.
//
// Logits come from router_tc.cu as ksplit partial sums; the selection kernel
// below adds them in a fixed order, so results are deterministic.
#include <math_constants.h>

#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace rt {
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per token; lane l holds expert g*32 + l of every group g.
__global__ void __launch_bounds__(256) select_kernel(const float* __restrict__ partial, int ksplit,
                                                     const float* __restrict__ bias, int T, int E, int n_group,
                                                     int topk_group, int top_k, int mode, int norm, float scaling,
                                                     int32_t* __restrict__ idx, int64_t* __restrict__ idx64,
                                                     float* __restrict__ w_out) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const float NEG = -CUDART_INF_F;
  float s[8], key[8], lg[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) lg[g] = 0.f;
  // The K-split partials are added in split order (fixed, deterministic); the
  // eight groups' loads of one split are independent, so they are issued
  // together.
#pragma unroll 4
  for (int k = 0; k < ksplit; ++k) {
    const float* pk = partial + (static_cast<size_t>(k) * T + t) * E + lane;
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g < n_group) lg[g] += __ldg(pk + g * 32);
  }
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    s[g] = NEG;
    key[g] = NEG;
    if (g < n_group) {
      const int e = g * 32 + lane;
      s[g] = 1.0f / (1.0f + expf(-lg[g]));
      key[g] = mode == 1 ? s[g] + __ldg(bias + e) : s[g];
    }
  }
  // group scores (identical in every lane)
  float gsc[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    gsc[g] = NEG;
    if (g < n_group) {
      const float m1 = warp_max(key[g]);
      if (mode == 1) {
        const unsigned at = __ballot_sync(0xffffffffu, key[g] == m1);
        const int first = __ffs(at) - 1;
        const float m2 = warp_max(lane == first ? NEG : key[g]);
        gsc[g] = m1 + m2;
      } else {
        gsc[g] = m1;
      }
    }
  }
  unsigned keep = 0;
  for (int r = 0; r < topk_group; ++r) {
    float best = NEG;
    int bi = -1;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g < n_group && !((keep >> g) & 1u) && (bi < 0 || gsc[g] > best)) {
        best = gsc[g];
        bi = g;
      }
    }
    keep |= 1u << bi;
  }
  float cand[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) cand[g] = ((keep >> g) & 1u) ? key[g] : (mode == 1 ? NEG : 0.0f);
  float topv[8], tops[8];
  int tope[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    topv[r] = 0.f;
    tops[r] = 0.f;
    tope[r] = 0;
    if (r < top_k) {
      // local best (lowest expert id among equals), then warp arg-max
      float v = NEG;
      int e = 0x7fffffff;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if (g < n_group && (cand[g] > v || (cand[g] == v && g * 32 + lane < e))) {
          v = cand[g];
          e = g * 32 + lane;
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oe = __shfl_xor_sync(0xffffffffu, e, o);
        if (ov > v || (ov == v && oe < e)) {
          v = ov;
          e = oe;
        }
      }
      float sv = 0.f;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        if (g == (e >> 5)) {
          sv = s[g];
          if (lane == (e & 31)) cand[g] = NEG;  // taken
        }
      }
      sv = __shfl_sync(0xffffffffu, sv, e & 31);
      topv[r] = v;
      tops[r] = sv;
      tope[r] = e;
    }
  }
  float sum = 0.f;
#pragma unroll
  for (int r = 0; r < 8; ++r)
    if (r < top_k) sum += mode == 1 ? tops[r] : topv[r];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    if (r < top_k && lane == r) {
      float wv;
      if (mode == 1) wv = tops[r] / sum * scaling;
      else wv = norm ? topv[r] / (sum + 1e-9f) : topv[r];
      idx[static_cast<size_t>(t) * top_k + r] = tope[r];
      if (idx64) idx64[static_cast<size_t>(t) * top_k + r] = tope[r];
      w_out[static_cast<size_t>(t) * top_k + r] = wv;
    }
  }
}
}  // namespace rt

cudaError_t launch_router_select(const float* partial, int ksplit, const float* bias, int T, int E, int n_group,
                                 int topk_group, int top_k, int mode, int norm, float scaling, int32_t* idx,
                                 int64_t* idx64, float* w, cudaStream_t stream) {
  const int blocks = (T * 32 + 255) / 256;
  rt::select_kernel<<<blocks, 256, 0, stream>>>(partial, ksplit, bias, T, E, n_group, topk_group, top_k, mode, norm,
                                                scaling, idx, idx64, w);
  return cudaGetLastError();
}

}  // namespace dsmoe
