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
// Logits: a split-K fp32 SIMT GEMM writes ksplit partial sums; the selection
// kernel adds them in a fixed order, so results are deterministic. Products of
// two bf16 values are exact in fp32, so the only difference from the
// reference's CPU matmul is the order of the fp32 additions.
#include <math_constants.h>

#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace rt {
constexpr int BT = 64;  // tokens per block
constexpr int BE = 64;  // experts per block
constexpr int BKR = 32;  // k per smem tile

__global__ void __launch_bounds__(256) logits_kernel(const __nv_bfloat16* __restrict__ x,
                                                     const __nv_bfloat16* __restrict__ gw,
                                                     float* __restrict__ partial, int T, int H, int E,
                                                     int k_per_split) {
  __shared__ __align__(16) float xs[BKR][BT + 4];
  __shared__ __align__(16) float gs[BKR][BE + 4];
  const int t0 = blockIdx.x * BT;
  const int e0 = blockIdx.y * BE;
  const int ks = blockIdx.z;
  const int kbeg = ks * k_per_split;
  const int kend = min(H, kbeg + k_per_split);
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int lr = tid >> 2, lk = (tid & 3) * 8;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = kbeg; k0 < kend; k0 += BKR) {
    uint4 xv = make_uint4(0, 0, 0, 0);
    if (t0 + lr < T) xv = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(t0 + lr) * H + k0 + lk));
    uint4 gv = make_uint4(0, 0, 0, 0);
    if (e0 + lr < E) gv = __ldg(reinterpret_cast<const uint4*>(gw + static_cast<size_t>(e0 + lr) * H + k0 + lk));
    const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&xv);
    const __nv_bfloat16* gb = reinterpret_cast<const __nv_bfloat16*>(&gv);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      xs[lk + i][lr] = __bfloat162float(xb[i]);
      gs[lk + i][lr] = __bfloat162float(gb[i]);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BKR; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[kk][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&gs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t < T && e0 + tx * 4 < E)
      *reinterpret_cast<float4*>(partial + (static_cast<size_t>(ks) * T + t) * E + e0 + tx * 4) =
          make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
}

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
  float s[8], key[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    s[g] = NEG;
    key[g] = NEG;
    if (g < n_group) {
      const int e = g * 32 + lane;
      float l = 0.f;
      for (int k = 0; k < ksplit; ++k) l += __ldg(partial + (static_cast<size_t>(k) * T + t) * E + e);
      s[g] = 1.0f / (1.0f + expf(-l));
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

int router_ksplit(int T, int H, int E, int num_sms) {
  const int k_tiles = H / rt::BKR;
  const int base = ((T + rt::BT - 1) / rt::BT) * ((E + rt::BE - 1) / rt::BE);
  if (base <= 0) return 1;
  int want = (2 * num_sms + base - 1) / base;
  if (want < 1) want = 1;
  int best = 1;
  for (int d = 1; d <= k_tiles && d <= 64; ++d)
    if (k_tiles % d == 0 && d <= want) best = d;
  return best;
}

cudaError_t launch_router_logits(const void* x, const void* gate, float* partial, int T, int H, int E, int ksplit,
                                 cudaStream_t stream) {
  const int kps = (H / rt::BKR / ksplit) * rt::BKR;
  dim3 grid((T + rt::BT - 1) / rt::BT, (E + rt::BE - 1) / rt::BE, ksplit);
  rt::logits_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                              static_cast<const __nv_bfloat16*>(gate), partial, T, H, E, kps);
  return cudaGetLastError();
}

cudaError_t launch_router_select(const float* partial, int ksplit, const float* bias, int T, int E, int n_group,
                                 int topk_group, int top_k, int mode, int norm, float scaling, int32_t* idx,
                                 int64_t* idx64, float* w, cudaStream_t stream) {
  const int blocks = (T * 32 + 255) / 256;
  rt::select_kernel<<<blocks, 256, 0, stream>>>(partial, ksplit, bias, T, E, n_group, topk_group, top_k, mode, norm,
                                                scaling, idx, idx64, w);
  return cudaGetLastError();
}

}  // namespace dsmoe
