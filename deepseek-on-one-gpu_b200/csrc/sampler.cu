// Temperature + nucleus (top-p) sampling of the next token, on the device.
//
// The reference samples each decode step on the host side of a per-token
// loop (inference/engine.py:166-190): softmax(logits / T), a full descending
// sort of the 129,280 probabilities, cumsum, mask every position whose
// preceding mass exceeds top_p, renormalise, torch.multinomial, then
// .item() to read the token back. This kernel does the same selection with
// no sort and no host round trip:
//
//   * one thread-block cluster per row; CTA c of the cluster holds logits
//     [c * 16384, (c + 1) * 16384) of the row in registers (16 order keys
//     per thread, 1024 threads), read from memory once;
//   * the order of the probabilities is the order of the logits (exp and the
//     division by T > 0 are monotonic), so elements are ranked by an
//     order-preserving 32-bit key of the logit itself;
//   * every probability becomes an exact integer mass q = round(e * 2^40),
//     e = exp(l / T - max / T); sums of masses are exact and independent of
//     the summation order, so every decision below is deterministic and
//     identical in all CTAs of the cluster;
//   * "the first position, in descending order, where the running mass
//     exceeds a target" is found by a radix select over the keys: four
//     passes of 8-bit digits, each a cluster-wide histogram of (mass, count)
//     per digit (warp-aggregated shared-memory atomics, the CTAs' histograms
//     summed through distributed shared memory), then a scan from the top
//     digit. Run with target floor(top_p * Q) it finds the last element of
//     the nucleus (the reference keeps a position iff the mass before it is
//     <= top_p); run with target floor(u * kept mass) it finds the sampled
//     element (inverse CDF in descending order, the order the reference's
//     multinomial indexes).
//   * equal logits are ordered by vocabulary index (a stable sort); the
//     reference's sort leaves their order unspecified.
//
// temperature == 0 is the reference's argmax (first maximal index, a NaN
// counting as the maximum). For temperature > 0, a row whose maximum logit is
// not finite (a NaN anywhere, or +-inf, where the reference's softmax yields
// NaN) gets token -1.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace dsmoe {

namespace smp {
constexpr int THREADS = 1024;
constexpr int WARPS = THREADS / 32;
constexpr int EPT = 16;                 // logits per thread
constexpr int CHUNK = THREADS * EPT;    // logits per CTA
constexpr int RADIX = 256;
constexpr float kMassScale = 1099511627776.0f;  // 2^40

struct Shared {
  unsigned long long hmass[3][RADIX];  // [0]: first-digit histogram (kept), [1], [2]: later passes, alternating
  unsigned int hcount[3][RADIX];
  unsigned long long scan_m[RADIX];    // cluster totals per digit, descending digit order, then scanned
  unsigned int scan_n[RADIX];
  unsigned long long warp64[WARPS];
  unsigned int warp32[WARPS];
  unsigned long long cta_max;          // read by the other CTAs of the cluster
  unsigned long long cta_mass;
  unsigned int cta_ties;
};

// Order-preserving key: a < b (as floats, -0 == +0 after canonicalisation)
// iff key(a) < key(b).
__device__ __forceinline__ uint32_t sort_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Key 0 marks positions past the end of the row (a real logit never gets it:
// NaNs are mapped to kNaNKey).
constexpr uint32_t kNoKey = 0u;
constexpr uint32_t kNaNKey = 0xffffffffu;

// Integer mass of a logit: round(2^40 * exp(l / T - max / T)), 0 past the
// end of the row. Written with explicitly rounded operations so that every
// evaluation, wherever it is inlined, gives the same bits.
__device__ __forceinline__ unsigned long long mass_of(uint32_t key, float temperature, float mt) {
  if (key == kNoKey) return 0ull;
  const float x = __fsub_rn(__fdiv_rn(key_value(key), temperature), mt);
  return __float2ull_rn(__fmul_rn(expf(x), kMassScale));
}

template <bool kMax>
__device__ __forceinline__ unsigned long long block_reduce(unsigned long long v, unsigned long long* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? (w > v ? w : v) : v + w;
  }
  __syncthreads();  // scratch free from its previous use
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  v = lane < WARPS ? scratch[lane] : 0ull;  // 0 is the identity of both (values are >= 0)
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMax ? (w > v ? w : v) : v + w;
  }
  return v;
}

// Exclusive prefix sum over the block's threads (in thread order); `total`
// receives the block sum.
__device__ __forceinline__ unsigned block_excl_scan(unsigned v, unsigned* scratch, unsigned& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned w = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += w;
  }
  __syncthreads();
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  const unsigned wsum = lane < WARPS ? scratch[lane] : 0u;
  unsigned wincl = wsum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned w = __shfl_up_sync(0xffffffffu, wincl, o);
    if (lane >= o) wincl += w;
  }
  total = __shfl_sync(0xffffffffu, wincl, 31);
  const unsigned warp_excl = __shfl_sync(0xffffffffu, wincl - wsum, warp);
  return warp_excl + incl - v;
}

// Adds (mass q, count 1) to digit `d` of the histogram for every lane with
// `pred`; lanes of a warp that share a digit are summed first, so one atomic
// per (warp, digit). q <= 2^40 is summed as two 20-bit halves (32 lanes of
// 2^20 fit 32 bits).
__device__ __forceinline__ void hist_add(bool pred, uint32_t d, unsigned long long q, unsigned long long* hm,
                                         unsigned* hc) {
  const unsigned act = __ballot_sync(0xffffffffu, pred);
  if (pred) {
    const unsigned grp = __match_any_sync(act, d);
    const unsigned lo = __reduce_add_sync(grp, static_cast<unsigned>(q & 0xfffffu));
    const unsigned hi = __reduce_add_sync(grp, static_cast<unsigned>(q >> 20));
    if ((threadIdx.x & 31) == static_cast<unsigned>(__ffs(grp) - 1)) {
      atomicAdd(&hm[d], (static_cast<unsigned long long>(hi) << 20) + lo);
      atomicAdd(&hc[d], static_cast<unsigned>(__popc(grp)));
    }
  }
}

// Histogram of the digit at `shift` over the elements with mass whose key
// matches `prefix` on the bits of `pmask` (the mass is only evaluated for
// matching elements).
__device__ __forceinline__ void accumulate(const uint32_t* key, float temperature, float mt, uint32_t prefix,
                                           uint32_t pmask, int shift, unsigned long long* hm, unsigned* hc) {
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const bool match = (key[i] & pmask) == prefix;
    const unsigned long long q = match ? mass_of(key[i], temperature, mt) : 0ull;
    hist_add(q != 0, (key[i] >> shift) & (RADIX - 1), q, hm, hc);
  }
}

struct Pick {
  uint32_t key;                 // key of the element found
  unsigned long long above;     // mass of all elements with a larger key
  unsigned n_above;             // their number
  unsigned ties;                // elements with exactly this key (all of equal mass)
  unsigned long long tie_mass;  // their total mass
};

// The element (key) at which the descending running mass first exceeds
// `target` (target < total mass). Uses the first-digit histogram hmass[0],
// built by the caller; later passes alternate between buffers 1 and 2
// (`flip`), so that a CTA never clears a histogram another CTA may still be
// reading (two cluster barriers separate a read from the next clear).
__device__ __forceinline__ Pick radix_select(unsigned long long target, const uint32_t* key, float temperature,
                                             float mt, Shared& s, cg::cluster_group& cluster, int ncta, int& flip) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  Pick p{0, 0, 0, 0, 0};
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    int buf = 0;
    if (pass > 0) {
      buf = 1 + flip;
      flip ^= 1;
      if (tid < RADIX) {
        s.hmass[buf][tid] = 0;
        s.hcount[buf][tid] = 0;
      }
      __syncthreads();
      accumulate(key, temperature, mt, prefix, pmask, shift, s.hmass[buf], s.hcount[buf]);
      cluster.sync();  // every CTA's histogram complete and visible
    }
    // Cluster totals per digit, digit 255 first (largest keys first).
    const int lane = tid & 31, warp = tid >> 5;
    unsigned long long m = 0;
    unsigned n = 0;
    if (tid < RADIX) {
      const int d = RADIX - 1 - tid;
      for (int r = 0; r < ncta; ++r) {
        m += cluster.map_shared_rank(&s.hmass[buf][0], r)[d];
        n += cluster.map_shared_rank(&s.hcount[buf][0], r)[d];
      }
      // inclusive scan within the warp, then across the 8 warps
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long wm = __shfl_up_sync(0xffffffffu, m, o);
        const unsigned wn = __shfl_up_sync(0xffffffffu, n, o);
        if (lane >= o) {
          m += wm;
          n += wn;
        }
      }
      if (lane == 31) {
        s.warp64[warp] = m;
        s.warp32[warp] = n;
      }
    }
    __syncthreads();
    if (tid < RADIX) {
      for (int w = 0; w < warp; ++w) {
        m += s.warp64[w];
        n += s.warp32[w];
      }
      s.scan_m[tid] = m;
      s.scan_n[tid] = n;
    }
    // The running mass is monotonic in tid, so the digits that cross the
    // target form a suffix; the first crossing one is RADIX - count.
    const bool over = tid < RADIX && p.above + m > target;
    int first = RADIX - __syncthreads_count(over);
    if (first >= RADIX) first = RADIX - 1;  // cannot happen for target < mass of the prefix
    const unsigned long long incl_m = s.scan_m[first];
    const unsigned incl_n = s.scan_n[first];
    const unsigned long long excl_m = first ? s.scan_m[first - 1] : 0ull;
    const unsigned excl_n = first ? s.scan_n[first - 1] : 0u;
    p.above += excl_m;
    p.n_above += excl_n;
    p.ties = incl_n - excl_n;
    p.tie_mass = incl_m - excl_m;
    prefix |= static_cast<uint32_t>(RADIX - 1 - first) << shift;
    pmask |= static_cast<uint32_t>(RADIX - 1) << shift;
    __syncthreads();  // scan_m / warp scratch reused by the next pass
  }
  p.key = prefix;
  return p;
}

__global__ void __launch_bounds__(THREADS, 1)
top_p_kernel(const float* __restrict__ logits, int V, long long ld, float temperature, float top_p,
             const float* __restrict__ uniforms, long long* __restrict__ tokens, int* __restrict__ nucleus) {
  __shared__ Shared s;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int ncta = static_cast<int>(cluster.num_blocks());
  const int row = blockIdx.y;
  const int tid = threadIdx.x;
  const float* src = logits + static_cast<size_t>(row) * static_cast<size_t>(ld);
  const int base = rank * CHUNK + tid * EPT;
  if (rank == 0 && tid == 0) tokens[row] = -1;

  uint32_t key[EPT];
  {
    float l[EPT];
    if (base + EPT <= V && (reinterpret_cast<uintptr_t>(src + base) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < EPT; i += 4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src + base + i));
        l[i] = v.x;
        l[i + 1] = v.y;
        l[i + 2] = v.z;
        l[i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPT; ++i) l[i] = base + i < V ? __ldg(src + base + i) : 0.f;
    }
    // -0 -> +0 so that equal logits get equal keys; every NaN (either sign)
    // gets the largest key, above +inf, as in torch's max / argmax
#pragma unroll
    for (int i = 0; i < EPT; ++i)
      key[i] = base + i >= V ? kNoKey : isnan(l[i]) ? kNaNKey : sort_key(__fadd_rn(l[i], 0.f));
  }

  // 1. maximum logit, first index among equal maxima
  unsigned long long best = 0;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const unsigned long long c = (static_cast<unsigned long long>(key[i]) << 32) |
                                 (0xffffffffu - static_cast<uint32_t>(base + i));
    if (key[i] != kNoKey && c > best) best = c;
  }
  best = block_reduce<true>(best, s.warp64);
  if (tid == 0) s.cta_max = best;
  cluster.sync();
  unsigned long long gbest = 0;
  for (int r = 0; r < ncta; ++r) {
    const unsigned long long c = *cluster.map_shared_rank(&s.cta_max, r);
    gbest = c > gbest ? c : gbest;
  }
  const float m = key_value(static_cast<uint32_t>(gbest >> 32));
  const long long argmax = static_cast<long long>(0xffffffffu - static_cast<uint32_t>(gbest & 0xffffffffu));
  if (temperature == 0.f || !isfinite(m)) {
    if (rank == 0 && tid == 0) {
      tokens[row] = temperature == 0.f ? argmax : -1;
      if (nucleus) nucleus[row] = temperature == 0.f ? 1 : 0;
    }
    cluster.sync();  // no CTA leaves while another may still read its shared memory
    return;
  }

  // 2. integer masses, their total Q, and the first-digit histogram
  const float mt = __fdiv_rn(m, temperature);
  unsigned long long qsum = 0;
#pragma unroll
  for (int i = 0; i < EPT; ++i) qsum += mass_of(key[i], temperature, mt);
  qsum = block_reduce<false>(qsum, s.warp64);
  if (tid == 0) s.cta_mass = qsum;
  if (tid < RADIX) {
    s.hmass[0][tid] = 0;
    s.hcount[0][tid] = 0;
  }
  __syncthreads();
  accumulate(key, temperature, mt, 0u, 0u, 24, s.hmass[0], s.hcount[0]);
  cluster.sync();
  unsigned long long Q = 0;
  for (int r = 0; r < ncta; ++r) Q += *cluster.map_shared_rank(&s.cta_mass, r);

  // 3. nucleus: keep a position iff the mass before it is <= top_p * Q
  int flip = 0;
  const unsigned long long tq =
      static_cast<unsigned long long>(floor(static_cast<double>(top_p) * static_cast<double>(Q)));
  unsigned long long kept_mass = Q;
  long long kept = V;
  if (Q > tq) {
    const Pick p = radix_select(tq, key, temperature, mt, s, cluster, ncta, flip);
    const unsigned long long q = p.ties && p.tie_mass ? p.tie_mass / p.ties : 1ull;  // ties >= 1, mass > 0
    unsigned long long k = (tq - p.above) / q + 1;
    if (k > p.ties) k = p.ties;
    kept_mass = p.above + k * q;
    kept = static_cast<long long>(p.n_above) + static_cast<long long>(k);
  }

  // 4. sample: the element where the descending running mass first exceeds
  //    u * kept mass
  float u = uniforms[row];
  if (!(u >= 0.f)) u = 0.f;
  unsigned long long t2 =
      static_cast<unsigned long long>(floor(static_cast<double>(u) * static_cast<double>(kept_mass)));
  if (t2 >= kept_mass) t2 = kept_mass - 1;
  const Pick p2 = radix_select(t2, key, temperature, mt, s, cluster, ncta, flip);
  const unsigned long long q2 = p2.ties && p2.tie_mass ? p2.tie_mass / p2.ties : 1ull;
  const unsigned j = static_cast<unsigned>((t2 - p2.above) / q2);  // which of the equal logits, in index order

  // 5. the j-th element (by vocabulary index) with the sampled key
  unsigned mine = 0;
#pragma unroll
  for (int i = 0; i < EPT; ++i) mine += key[i] == p2.key ? 1u : 0u;
  unsigned cta_total;
  const unsigned excl = block_excl_scan(mine, s.warp32, cta_total);
  if (tid == 0) s.cta_ties = cta_total;
  cluster.sync();
  unsigned off = 0;
  for (int r = 0; r < rank; ++r) off += *cluster.map_shared_rank(&s.cta_ties, r);
  if (j >= off + excl && j < off + excl + mine) {
    unsigned want = j - off - excl;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      if (key[i] == p2.key) {
        if (want == 0) tokens[row] = base + i;
        --want;
      }
    }
  }
  if (rank == 0 && tid == 0 && nucleus) nucleus[row] = static_cast<int>(kept);
  cluster.sync();
}
}  // namespace smp

int top_p_max_vocab() { return 8 * smp::CHUNK; }

cudaError_t launch_top_p(const float* logits, int rows, int V, long long ld, float temperature, float top_p,
                         const float* uniforms, long long* tokens, int* nucleus, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int ncta = (V + smp::CHUNK - 1) / smp::CHUNK;
  if (V <= 0 || ncta > 8 || rows > 65535) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ncta);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(ncta), static_cast<unsigned>(rows), 1);
  cfg.blockDim = dim3(smp::THREADS, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, smp::top_p_kernel, logits, V, ld, temperature, top_p, uniforms, tokens, nucleus);
}

}  // namespace dsmoe
