// K2: token permutation by expert, fused with the FP8 hi/lo activation split.
//
// The reference loops over tokens and runs each token's 8 experts one at a
// time (inference/forward.py:140-151). Here tokens are grouped by expert so
// that each expert's weights are read once for all of its tokens:
//   count   histogram of (token, k) pairs per expert group
//   plan    exclusive scans -> 32-row-aligned segment starts, work-unit starts
//           of both GEMMs (one block)
//   scatter one CTA per token: claims one row in each of its experts'
//           segments (+ its row in the shared-expert segment), splits the bf16
//           row into hi/lo e4m3 terms with one fp32 scale per row, writes the
//           row copies and records the (token, k) -> row map used by the
//           combine.
// Activation format (per row r):
//   sx = amax / 448;  q = x * 448 / amax;  hi = e4m3(q);  lo = e4m3(q - hi)
//   x ~= (hi + lo) * sx   (about 8 significant bits instead of 4; one scale
//   per row gives the same error as one per 128 columns, and lets the GEMM
//   apply it once after the K loop).
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace pm {
constexpr int MAX_GROUPS = 512;

// n_rows (optional): the row count on the device; only its first
// n_rows * per_row pairs are counted (n_pairs is the bound the grid covers).
__global__ void __launch_bounds__(256) count_kernel(const int32_t* __restrict__ idx, int n_pairs,
                                                    int32_t* __restrict__ counts, int n_groups,
                                                    const int32_t* __restrict__ n_rows, int per_row) {
  __shared__ int hist[MAX_GROUPS];
  for (int i = threadIdx.x; i < n_groups; i += blockDim.x) hist[i] = 0;
  if (n_rows) n_pairs = min(n_pairs, *n_rows * per_row);
  __syncthreads();
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n_pairs; p += gridDim.x * blockDim.x) {
    const int g = idx[p] + 1;
    if (g >= 1 && g < n_groups) atomicAdd(&hist[g], 1);
  }
  __syncthreads();
  for (int i = 1 + threadIdx.x; i < n_groups; i += blockDim.x)
    if (hist[i]) atomicAdd(&counts[i], hist[i]);
}

template <int N>
__device__ __forceinline__ int block_excl_scan(int v, int* buf) {
  // Hillis-Steele inclusive scan over blockDim.x == N entries, then shift.
  const int i = threadIdx.x;
  buf[i] = v;
  __syncthreads();
  for (int o = 1; o < N; o <<= 1) {
    const int add = i >= o ? buf[i - o] : 0;
    __syncthreads();
    buf[i] += add;
    __syncthreads();
  }
  const int incl = buf[i];
  __syncthreads();
  return incl - v;
}

__global__ void __launch_bounds__(MAX_GROUPS) plan_kernel(int32_t* __restrict__ counts, int n_groups,
                                                          int shared_tokens, int tile, int mt_up, int mt_dn,
                                                          int32_t* __restrict__ row_start,
                                                          int32_t* __restrict__ cursor,
                                                          int32_t* __restrict__ ustart_up,
                                                          int32_t* __restrict__ ustart_dn) {
  __shared__ int buf[MAX_GROUPS];
  const int i = threadIdx.x;
  int c = 0;
  if (i < n_groups) c = i == 0 ? shared_tokens : counts[i];
  __syncthreads();
  if (i == 0) counts[0] = shared_tokens;
  const int nt = (c + tile - 1) / tile;
  const int seg = block_excl_scan<MAX_GROUPS>((c + 31) & ~31, buf);
  const int uu = block_excl_scan<MAX_GROUPS>(mt_up * nt, buf);
  const int ud = block_excl_scan<MAX_GROUPS>(mt_dn * nt, buf);
  if (i <= n_groups) {
    row_start[i] = seg;
    if (ustart_up) ustart_up[i] = uu;
    if (ustart_dn) ustart_dn[i] = ud;
  }
  if (i < n_groups) cursor[i] = 0;
}

// hi/lo split of 8 values (already multiplied by 448 / amax), packed.
__device__ __forceinline__ void split8(const uint4 v, float inv, uint2& hv, uint2& lv) {
  const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v);
  uint32_t hw[2], lw[2];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float q0 = __bfloat162float(vb[i]) * inv, q1 = __bfloat162float(vb[i + 1]) * inv;
    const uint16_t h2 = f32x2_to_e4m3x2(q0, q1);
    const uint16_t l2 = f32x2_to_e4m3x2(q0 - e4m3_to_f32(static_cast<uint8_t>(h2 & 0xff)),
                                        q1 - e4m3_to_f32(static_cast<uint8_t>(h2 >> 8)));
    if ((i & 2) == 0) {
      hw[i >> 2] = h2;
      lw[i >> 2] = l2;
    } else {
      hw[i >> 2] |= static_cast<uint32_t>(h2) << 16;
      lw[i >> 2] |= static_cast<uint32_t>(l2) << 16;
    }
  }
  hv = make_uint2(hw[0], hw[1]);
  lv = make_uint2(lw[0], lw[1]);
}

__device__ __forceinline__ float amax8(const uint4 v, float m) {
  const __nv_bfloat16* vb = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(__bfloat162float(vb[i])));
  return m;
}

// One CTA of QS_THREADS per token: the token's rows are placed (one atomic
// per routed expert), its row amax is reduced over the CTA, and its hi/lo
// split is written to every row it occupies (the shared-expert row and one
// per routed expert). Rows of up to QS_THREADS * 8 * QS_MAXC columns stay in
// registers between the two passes; wider rows are read twice.
constexpr int QS_THREADS = 256;
constexpr int QS_MAXC = 4;

__global__ void __launch_bounds__(QS_THREADS) quant_scatter_kernel(const __nv_bfloat16* __restrict__ x, int T, int H,
                                                                   const int32_t* __restrict__ idx, int top_k,
                                                                   int n_groups, int has_shared,
                                                                   const int32_t* __restrict__ row_start,
                                                                   int32_t* __restrict__ cursor, int P,
                                                                   uint8_t* __restrict__ xq, float* __restrict__ sx,
                                                                   int32_t* __restrict__ pos,
                                                                   const int32_t* __restrict__ n_rows) {
  const int t = blockIdx.x;
  if (n_rows && t >= *n_rows) return;  // rows beyond the device-side count (whole CTA)
  __shared__ int s_rows[9];
  __shared__ float s_red[QS_THREADS / 32];
  const int tid = threadIdx.x;
  if (tid < top_k) {
    const int g = idx[static_cast<size_t>(t) * top_k + tid] + 1;  // entries < 0 (no expert) are skipped
    int myrow = -1;
    if (g >= 1 && g < n_groups) myrow = row_start[g] + atomicAdd(&cursor[g], 1);
    pos[static_cast<size_t>(t) * top_k + tid] = myrow;
    s_rows[has_shared + tid] = myrow;
  }
  if (tid == 0 && has_shared) s_rows[0] = row_start[0] + t;
  const int n = has_shared + top_k;
  const __nv_bfloat16* xr = x + static_cast<size_t>(t) * H;
  const uint4* xv = reinterpret_cast<const uint4*>(xr);
  const int nchunks = H / 8;
  const bool in_regs = nchunks <= QS_THREADS * QS_MAXC;
  uint4 v[QS_MAXC];
  float amax = 0.f;
  if (in_regs) {
#pragma unroll
    for (int i = 0; i < QS_MAXC; ++i) {
      const int c = tid + i * QS_THREADS;
      if (c < nchunks) {
        v[i] = __ldg(xv + c);
        amax = amax8(v[i], amax);
      }
    }
  } else {
    for (int c = tid; c < nchunks; c += QS_THREADS) amax = amax8(__ldg(xv + c), amax);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((tid & 31) == 0) s_red[tid >> 5] = amax;
  __syncthreads();  // also publishes s_rows
  amax = s_red[0];
#pragma unroll
  for (int i = 1; i < QS_THREADS / 32; ++i) amax = fmaxf(amax, s_red[i]);
  const float inv = amax > 0.f ? 448.f / amax : 0.f;
  int rows[9];
#pragma unroll
  for (int r = 0; r < 9; ++r) rows[r] = r < n ? s_rows[r] : -1;
  if (tid < n) {
    const int rr = s_rows[tid];
    if (rr >= 0) sx[rr] = amax / 448.f;
  }
  uint8_t* xq_lo = xq + static_cast<size_t>(P) * H;
  auto write = [&](int c, const uint4& val) {
    uint2 hv, lv;
    split8(val, inv, hv, lv);
    const int col = c * 8;
#pragma unroll
    for (int r = 0; r < 9; ++r) {
      if (rows[r] >= 0) {
        const size_t off = static_cast<size_t>(rows[r]) * H + col;
        *reinterpret_cast<uint2*>(xq + off) = hv;
        *reinterpret_cast<uint2*>(xq_lo + off) = lv;
      }
    }
  };
  if (in_regs) {
#pragma unroll
    for (int i = 0; i < QS_MAXC; ++i) {
      const int c = tid + i * QS_THREADS;
      if (c < nchunks) write(c, v[i]);
    }
  } else {
    for (int c = tid; c < nchunks; c += QS_THREADS) write(c, __ldg(xv + c));
  }
}
}  // namespace pm

cudaError_t launch_count(const int32_t* idx, int n_pairs, int32_t* counts, int n_groups, cudaStream_t stream,
                         const int32_t* n_rows, int per_row) {
  if (n_groups > pm::MAX_GROUPS) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * n_groups, stream);
  if (e != cudaSuccess) return e;
  if (n_pairs == 0) return cudaSuccess;
  int blocks = (n_pairs + 255) / 256;
  if (blocks > 296) blocks = 296;
  pm::count_kernel<<<blocks, 256, 0, stream>>>(idx, n_pairs, counts, n_groups, n_rows, per_row);
  return cudaGetLastError();
}

cudaError_t launch_plan(int32_t* counts, int n_groups, int shared_tokens, int tile, int mt_up, int mt_dn,
                        int32_t* row_start, int32_t* cursor, int32_t* ustart_up, int32_t* ustart_dn,
                        cudaStream_t stream) {
  if (n_groups + 1 > pm::MAX_GROUPS) return cudaErrorInvalidValue;
  pm::plan_kernel<<<1, pm::MAX_GROUPS, 0, stream>>>(counts, n_groups, shared_tokens, tile, mt_up, mt_dn, row_start,
                                                    cursor, ustart_up, ustart_dn);
  return cudaGetLastError();
}

cudaError_t launch_quant_scatter(const void* x, int T, int H, const int32_t* idx, int top_k, int n_groups,
                                 int has_shared, const int32_t* row_start, int32_t* cursor, int P, uint8_t* xq,
                                 float* sx, int32_t* pos, cudaStream_t stream, const int32_t* n_rows) {
  if (T == 0) return cudaSuccess;
  if (top_k + has_shared > 9) return cudaErrorInvalidValue;
  pm::quant_scatter_kernel<<<T, pm::QS_THREADS, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), T, H, idx,
                                                              top_k, n_groups, has_shared, row_start, cursor, P, xq,
                                                              sx, pos, n_rows);
  return cudaGetLastError();
}

}  // namespace dsmoe
