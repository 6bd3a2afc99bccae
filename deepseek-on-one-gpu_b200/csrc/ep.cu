// Expert parallelism: dispatch planning / packing and the final combine.
//
// With W ranks, rank d owns routed experts [d*El, (d+1)*El), El = E / W; the
// gate and the shared expert are replicated. A token is sent ONCE to every
// rank that owns at least one of its top-k experts (not once per expert), with
// the list of its experts on that rank (local ids, top-k order, -1 elsewhere)
// and their routing weights. The receiving rank returns one pre-reduced row
// per received token (sum over its experts, bf16 in top-k order), and the
// sending rank adds the returned rows in rank order:
//     out[t] = bf16(shared[t] + bf16(scale * acc)),  acc = bf16 sum over ranks
// which is the reference's bf16 combine (inference/forward.py:151-153) with
// the per-token sum regrouped by owning rank.
//
// Send buffer layout (what all-to-all moves): rows grouped by destination rank
// in rank order, inside a destination by token id. tok_rows[t][d] is the row
// of token t's copy for rank d (-1 if none), used by the combine.
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace ep {
constexpr int MAX_WORLD = 64;

__device__ __forceinline__ bool sends_to(const int64_t* idx, int t, int K, int El, int d) {
  for (int k = 0; k < K; ++k) {
    const int64_t e = idx[static_cast<size_t>(t) * K + k];
    if (e >= 0 && e / El == d) return true;
  }
  return false;
}

// One block per destination rank: how many tokens go there.
__global__ void __launch_bounds__(1024) count_kernel(const int64_t* __restrict__ idx, int T, int K, int El,
                                                     int32_t* __restrict__ counts) {
  const int d = blockIdx.x;
  int c = 0;
  for (int t = threadIdx.x; t < T; t += blockDim.x) c += sends_to(idx, t, K, El, d);
  __shared__ int red[32];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x < 32) {
    int v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) counts[d] = v;
  }
}

// One block per destination rank: place its tokens (in token order) at
// offset(d) + rank-within-d, writing the routing list and the row map.
__global__ void __launch_bounds__(1024) place_kernel(const int64_t* __restrict__ idx, const float* __restrict__ w,
                                                     int T, int K, int El, int W,
                                                     const int32_t* __restrict__ counts,
                                                     int32_t* __restrict__ tok_rows, int32_t* __restrict__ send_tok,
                                                     int32_t* __restrict__ send_idx, float* __restrict__ send_w) {
  const int d = blockIdx.x;
  __shared__ int s_off;
  __shared__ int warp_sums[32];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int i = 0; i < d; ++i) o += counts[i];
    s_off = o;
  }
  __syncthreads();
  int base = s_off;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    const bool f = t < T && sends_to(idx, t, K, El, d);
    // block-wide exclusive scan of f
    const unsigned m = __ballot_sync(0xffffffffu, f);
    const int in_warp = __popc(m & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[wid] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int i = 0; i < nw; ++i) {
      const int v = warp_sums[i];
      if (i < wid) before += v;
      total += v;
    }
    if (t < T) {
      if (f) {
        const int row = base + before + in_warp;
        tok_rows[static_cast<size_t>(t) * W + d] = row;
        send_tok[row] = t;
        for (int k = 0; k < K; ++k) {
          const int64_t e = idx[static_cast<size_t>(t) * K + k];
          const bool mine = e >= 0 && e / El == d;
          send_idx[static_cast<size_t>(row) * K + k] = mine ? static_cast<int32_t>(e - static_cast<int64_t>(d) * El) : -1;
          send_w[static_cast<size_t>(row) * K + k] = mine ? w[static_cast<size_t>(t) * K + k] : 0.f;
        }
      } else {
        tok_rows[static_cast<size_t>(t) * W + d] = -1;
      }
    }
    base += total;
    __syncthreads();
  }
}

// send_x[s] = x[send_tok[s]]  (one block per row, 16-byte vectors)
__global__ void __launch_bounds__(256) gather_kernel(const __nv_bfloat16* __restrict__ x, int H,
                                                     const int32_t* __restrict__ send_tok,
                                                     const int32_t* __restrict__ counts, int W,
                                                     __nv_bfloat16* __restrict__ send_x) {
  __shared__ int s_total;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int i = 0; i < W; ++i) n += counts[i];
    s_total = n;
  }
  __syncthreads();
  for (int s = blockIdx.x; s < s_total; s += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(send_tok[s]) * H);
    uint4* dst = reinterpret_cast<uint4*>(send_x + static_cast<size_t>(s) * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = __ldg(src + c);
  }
}

// Peer-memory dispatch (one kernel instead of a local pack + all-to-all):
// every send row r of this rank (grouped by destination d, position k inside
// d's group) is written straight into rank d's receive buffers over NVLink,
// at row p = (rows that lower ranks send to d) + k, with its routing list and
// its origin (this rank, k); tok_rows is rewritten to d * cap + k, the row of
// the partial that d will store back into this rank's return buffer.
// counts_all[s][d] (all ranks' send counts, gathered beforehand) gives both
// offsets. Rows are 16-byte vectors; the kernel ends with a system fence.
__global__ void __launch_bounds__(256) push_kernel(const __nv_bfloat16* __restrict__ x, int H, int K, int W, int me,
                                                   int cap, const int32_t* __restrict__ counts_all,
                                                   const int32_t* __restrict__ send_tok,
                                                   const int32_t* __restrict__ send_idx,
                                                   const float* __restrict__ send_w, int32_t* __restrict__ tok_rows,
                                                   const uint64_t* __restrict__ recv_x,
                                                   const uint64_t* __restrict__ recv_meta, int* __restrict__ status) {
  __shared__ int s_lbase[MAX_WORLD + 1];  // this rank's rows before destination d
  __shared__ int s_rbase[MAX_WORLD];      // rows lower ranks send to d
  if (threadIdx.x == 0) {
    int o = 0;
    for (int d = 0; d < W; ++d) {
      s_lbase[d] = o;
      o += counts_all[me * W + d];
      int rb = 0;
      for (int s = 0; s < me; ++s) rb += counts_all[s * W + d];
      s_rbase[d] = rb;
    }
    s_lbase[W] = o;
  }
  __syncthreads();
  const int total = s_lbase[W];
  const size_t cap_rows = static_cast<size_t>(W) * cap;
  for (int r = blockIdx.x; r < total; r += gridDim.x) {
    int d = 0;
    while (d + 1 < W && s_lbase[d + 1] <= r) ++d;
    const int k = r - s_lbase[d];
    const size_t p = static_cast<size_t>(s_rbase[d]) + k;
    const int t = send_tok[r];
    if (k >= cap || p >= cap_rows) {
      // counts inconsistent with the buffers: write nothing, drop the row from
      // the combine and record the error
      if (threadIdx.x == 0) {
        tok_rows[static_cast<size_t>(t) * W + d] = -1;
        if (status) atomicCAS(status, 0, kDevBadCount);
      }
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<size_t>(t) * H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(recv_x[d]) + p * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = __ldg(src + c);
    // routing list: idx [W*cap][K] | weights [W*cap][K] | origin [W*cap][2]
    int32_t* meta = reinterpret_cast<int32_t*>(recv_meta[d]);
    if (threadIdx.x < K) {
      meta[p * K + threadIdx.x] = send_idx[static_cast<size_t>(r) * K + threadIdx.x];
      meta[cap_rows * K + p * K + threadIdx.x] = __float_as_int(send_w[static_cast<size_t>(r) * K + threadIdx.x]);
    } else if (threadIdx.x == K) {
      meta[2 * cap_rows * K + p * 2] = me;
      meta[2 * cap_rows * K + p * 2 + 1] = k;
      tok_rows[static_cast<size_t>(t) * W + d] = d * cap + k;
    }
  }
  __threadfence_system();
}

// Rows this rank receives in a peer-memory step: sum over source ranks s of
// counts_all[s][me] (one warp).
__global__ void recv_rows_kernel(const int32_t* __restrict__ counts_all, int W, int me, int32_t* __restrict__ out) {
  int v = 0;
  for (int s = threadIdx.x; s < W; s += 32) v += counts_all[s * W + me];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (threadIdx.x == 0) *out = v;
}

// out[t] = bf16(shared[t] + bf16(scale * acc)), acc = bf16 sum of the
// returned rows of token t in rank order.
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ part,
                                                      const int32_t* __restrict__ tok_rows, int W, int H,
                                                      const __nv_bfloat16* __restrict__ shared, float scale,
                                                      __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  __shared__ int s_row[MAX_WORLD];
  for (int d = threadIdx.x; d < W; d += blockDim.x) s_row[d] = tok_rows[static_cast<size_t>(t) * W + d];
  __syncthreads();
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int d = 0; d < W; ++d) {
      const int r = s_row[d];
      if (r < 0) continue;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(part + static_cast<size_t>(r) * H) + c);
      const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = bf16_round(acc[i] + __bfloat162float(vb[i]));
    }
    const uint4 sv = __ldg(reinterpret_cast<const uint4*>(shared + static_cast<size_t>(t) * H) + c);
    const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(&sv);
    uint4 o;
    __nv_bfloat16* ob = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) ob[i] = __float2bfloat16_rn(__bfloat162float(sb[i]) + bf16_round(acc[i] * scale));
    reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H)[c] = o;
  }
}
}  // namespace ep

cudaError_t launch_ep_dispatch(const int64_t* idx, const float* w, const void* x, int T, int K, int H, int W, int El,
                               int32_t* counts, int32_t* tok_rows, int32_t* send_tok, int32_t* send_idx,
                               float* send_w, void* send_x, cudaStream_t stream) {
  if (W < 1 || W > ep::MAX_WORLD) return cudaErrorInvalidValue;
  ep::count_kernel<<<W, 1024, 0, stream>>>(idx, T, K, El, counts);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  ep::place_kernel<<<W, 1024, 0, stream>>>(idx, w, T, K, El, W, counts, tok_rows, send_tok, send_idx, send_w);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  int blocks = T * (K < W ? K : W);
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  ep::gather_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), H, send_tok, counts, W,
                                                static_cast<__nv_bfloat16*>(send_x));
  return cudaGetLastError();
}

cudaError_t launch_ep_plan(const int64_t* idx, const float* w, int T, int K, int W, int El, int32_t* counts,
                           int32_t* tok_rows, int32_t* send_tok, int32_t* send_idx, float* send_w, cudaStream_t stream) {
  if (W < 1 || W > ep::MAX_WORLD) return cudaErrorInvalidValue;
  ep::count_kernel<<<W, 1024, 0, stream>>>(idx, T, K, El, counts);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  ep::place_kernel<<<W, 1024, 0, stream>>>(idx, w, T, K, El, W, counts, tok_rows, send_tok, send_idx, send_w);
  return cudaGetLastError();
}

cudaError_t launch_ep_push(const void* x, int T, int H, int K, int W, int me, int cap, const int32_t* counts_all,
                           const int32_t* send_tok, const int32_t* send_idx, const float* send_w, int32_t* tok_rows,
                           const uint64_t* recv_x, const uint64_t* recv_meta, int* status, int max_blocks,
                           cudaStream_t stream) {
  if (W < 1 || W > ep::MAX_WORLD || me < 0 || me >= W || K > 8) return cudaErrorInvalidValue;
  int blocks = T * (K < W ? K : W);
  if (blocks > 4096) blocks = 4096;
  if (max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  ep::push_kernel<<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), H, K, W, me, cap, counts_all,
                                              send_tok, send_idx, send_w, tok_rows, recv_x, recv_meta, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_recv_rows(const int32_t* counts_all, int W, int me, int32_t* out, cudaStream_t stream) {
  if (W < 1 || W > ep::MAX_WORLD || me < 0 || me >= W) return cudaErrorInvalidValue;
  ep::recv_rows_kernel<<<1, 32, 0, stream>>>(counts_all, W, me, out);
  return cudaGetLastError();
}

cudaError_t launch_ep_combine(const void* part, const int32_t* tok_rows, int T, int W, int H, const void* shared,
                              float scale, void* out, cudaStream_t stream) {
  if (T == 0) return cudaSuccess;
  if (W < 1 || W > ep::MAX_WORLD) return cudaErrorInvalidValue;
  ep::combine_kernel<<<T, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(part), tok_rows, W, H,
                                            static_cast<const __nv_bfloat16*>(shared), scale,
                                            static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

}  // namespace dsmoe
