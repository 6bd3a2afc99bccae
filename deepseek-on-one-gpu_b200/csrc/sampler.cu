// Temperature + nucleus (top-p) sampling of the next token, on the device.
//
// The reference samples each decode step on the host side of a per-token
// loop (inference/engine.py:166-190): softmax(logits / T), a full descending
// sort of the 129,280 probabilities, cumsum, mask every position whose
// preceding mass exceeds top_p, renormalise, torch.multinomial, then
// .item() to read the token back. This kernel does the same selection with
// no full sort and no host round trip:
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
//   * "the first element, in descending order, where the running mass
//     exceeds a target" is found in two levels. First a cluster-wide
//     histogram of (mass, count) over 1024 buckets of (max - l) / T (equal
//     widths over the 28.5 units in which an element has non-zero mass),
//     built once per row and scanned from the top bucket, gives the bucket
//     that crosses the target. Then the keys of that bucket (a few hundred
//     for real or random logits) are gathered from all CTAs through
//     distributed shared memory and every CTA finishes on them alone, with a
//     4-pass 8-bit radix select in its own shared memory. A bucket of more
//     than 4096 elements (rows of many equal logits) is resolved instead by
//     cluster-wide radix passes restricted to the bucket.
//   * With target floor(top_p * Q) this finds the last element of the
//     nucleus (the reference keeps a position iff the mass before it is
//     <= top_p); with target floor(u * kept mass) it finds the sampled
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
constexpr int MAX_CTAS = 8;             // CTAs per cluster (one row)
constexpr int RADIX = 256;              // digits of a key radix pass
constexpr int NCOPY = 8;                // histogram copies of a cluster radix pass (warp w -> copy w % NCOPY)
constexpr int VB = 1024;                // value buckets of the first level (one per thread)
constexpr int VCOPY = 4;                // copies of the value histogram
constexpr int CAP = 4096;               // keys a bucket may hold to be finished locally
constexpr float kMassScale = 1099511627776.0f;  // 2^40
// e = exp(x) has a non-zero mass round(e * 2^40) iff x > -28.42; buckets span 28.5
constexpr float kBucketScale = static_cast<float>(VB) / 28.5f;
static_assert(VB == THREADS, "one value bucket per thread");

struct Shared {
  // first level: value buckets (this CTA's histogram is read by the cluster)
  unsigned long long vpm[VCOPY][VB];
  unsigned int vpc[VCOPY][VB];
  unsigned long long vmass[VB];
  unsigned int vcount[VB];
  // second level: the crossing bucket's keys; one list per select (this
  // CTA's, read by the cluster) and the merged list of the whole cluster
  uint32_t cand[2][CAP];
  uint32_t merged[CAP];
  unsigned int cand_n[2];
  // key radix passes (local finish, and the cluster fallback)
  unsigned long long pm[NCOPY][RADIX];
  unsigned int pc[NCOPY][RADIX];
  unsigned long long hmass[2][RADIX];  // cluster fallback: this CTA's histogram, alternating
  unsigned int hcount[2][RADIX];
  // block scans and reductions
  unsigned long long scan_m[VB];
  unsigned int scan_n[VB];
  unsigned long long warp64[WARPS];
  unsigned int warp32[WARPS];
  unsigned long long cta_max;  // read by the other CTAs of the cluster
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

// x - max(x) for x = l / T, written with explicitly rounded operations so that
// every evaluation, wherever it is inlined, gives the same bits.
__device__ __forceinline__ float rel_x(uint32_t key, float temperature, float mt) {
  return __fsub_rn(__fdiv_rn(key_value(key), temperature), mt);
}

// Integer mass of a logit: round(2^40 * exp(l / T - max / T)), 0 past the end
// of the row.
__device__ __forceinline__ unsigned long long mass_of(uint32_t key, float temperature, float mt) {
  if (key == kNoKey) return 0ull;
  return __float2ull_rn(__fmul_rn(expf(rel_x(key, temperature, mt)), kMassScale));
}

// First-level bucket: 0 holds the largest logits; monotone in the key.
__device__ __forceinline__ int vbucket(uint32_t key, float temperature, float mt) {
  const float d = __fmul_rn(-rel_x(key, temperature, mt), kBucketScale);  // >= 0
  return d >= static_cast<float>(VB - 1) ? VB - 1 : static_cast<int>(d);
}

// Block-wide sum (kMax = false) or max of a 64-bit value; every thread gets
// the result.
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

// Sum of q over the lanes of `grp` (q <= 2^40, summed as two 20-bit halves:
// 32 lanes of 2^20 fit 32 bits); called by exactly the lanes of grp.
__device__ __forceinline__ unsigned long long group_sum(unsigned grp, unsigned long long q) {
  const unsigned lo = __reduce_add_sync(grp, static_cast<unsigned>(q & 0xfffffu));
  const unsigned hi = __reduce_add_sync(grp, static_cast<unsigned>(q >> 20));
  return (static_cast<unsigned long long>(hi) << 20) + lo;
}

// True (in every lane) when all lanes with `pred` share the digit `d`.
__device__ __forceinline__ bool warp_uniform(unsigned act, bool pred, uint32_t d) {
  const uint32_t d0 = __shfl_sync(0xffffffffu, d, __ffs(act) - 1);
  return __all_sync(0xffffffffu, !pred || d == d0);
}

// Adds (mass q, count 1) to digit `d` of the histogram for every lane with
// `pred`; lanes of a warp that share a digit are summed first, so one atomic
// per (warp, digit). Every lane of the warp must call it.
__device__ __forceinline__ void hist_add(bool pred, uint32_t d, unsigned long long q, unsigned long long* hm,
                                         unsigned* hc) {
  const unsigned act = __ballot_sync(0xffffffffu, pred);
  if (!act) return;  // warp-uniform
  const bool uni = warp_uniform(act, pred, d);
  if (pred) {
    const unsigned grp = uni ? act : __match_any_sync(act, d);
    const unsigned long long sum = group_sum(grp, q);
    if ((threadIdx.x & 31) == static_cast<unsigned>(__ffs(grp) - 1)) {
      atomicAdd(&hm[d], sum);
      atomicAdd(&hc[d], static_cast<unsigned>(__popc(grp)));
    }
  }
}

struct Pick {
  uint32_t key;                 // key of the element found
  unsigned long long above;     // mass of all elements with a larger key
  unsigned n_above;             // their number
  unsigned ties;                // elements with exactly this key (all of equal mass)
  unsigned long long tie_mass;  // their total mass
};

// Inclusive scan of the (mass, count) pairs held by threads tid < n (n a
// multiple of 32, <= THREADS), in thread order, then the first position whose
// running mass plus `base` exceeds `target`. Returns the position and, through
// the references, the sums before it and the pair at it. Every thread must
// call it.
__device__ __forceinline__ int scan_cross(unsigned long long m, unsigned c, int n, unsigned long long base,
                                          unsigned long long target, Shared& s, unsigned long long& excl_m,
                                          unsigned& excl_n, unsigned long long& own_m, unsigned& own_n) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < n) {  // whole warps
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long wm = __shfl_up_sync(0xffffffffu, m, o);
      const unsigned wc = __shfl_up_sync(0xffffffffu, c, o);
      if (lane >= o) {
        m += wm;
        c += wc;
      }
    }
  }
  __syncthreads();  // warp scratch free
  if (tid < n && lane == 31) {
    s.warp64[warp] = m;
    s.warp32[warp] = c;
  }
  __syncthreads();
  if (tid < n) {
    for (int w = 0; w < warp; ++w) {
      m += s.warp64[w];
      c += s.warp32[w];
    }
    s.scan_m[tid] = m;
    s.scan_n[tid] = c;
  }
  // the running mass is monotonic in the position: the crossing ones are a suffix
  const bool over = tid < n && base + m > target;
  int first = n - __syncthreads_count(over);
  if (first >= n) first = n - 1;  // cannot happen for target < base + total
  excl_m = first ? s.scan_m[first - 1] : 0ull;
  excl_n = first ? s.scan_n[first - 1] : 0u;
  own_m = s.scan_m[first] - excl_m;
  own_n = s.scan_n[first] - excl_n;
  __syncthreads();  // scan arrays reused by the next scan
  return first;
}

// Local finish: radix select over the n keys of s.merged (one value bucket),
// in this CTA's shared memory only.
__device__ __forceinline__ Pick local_select(int n, unsigned long long target, float temperature, float mt,
                                             Shared& s) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  Pick p{0, 0, 0, 0, 0};
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (tid < RADIX) {
      s.pm[0][tid] = 0;
      s.pc[0][tid] = 0;
    }
    __syncthreads();
    for (int b = 0; b < n; b += THREADS) {  // uniform trip count: every lane reaches hist_add
      const int i = b + tid;
      const uint32_t k = i < n ? s.merged[i] : kNoKey;
      const bool match = i < n && (k & pmask) == prefix;
      hist_add(match, (k >> shift) & (RADIX - 1), match ? mass_of(k, temperature, mt) : 0ull, s.pm[0], s.pc[0]);
    }
    __syncthreads();
    unsigned long long m = 0, em, om;
    unsigned c = 0, en, on;
    if (tid < RADIX) {
      m = s.pm[0][RADIX - 1 - tid];  // largest digit first
      c = s.pc[0][RADIX - 1 - tid];
    }
    const int first = scan_cross(m, c, RADIX, p.above, target, s, em, en, om, on);
    p.above += em;
    p.n_above += en;
    p.ties = on;
    p.tie_mass = om;
    prefix |= static_cast<uint32_t>(RADIX - 1 - first) << shift;
    pmask |= static_cast<uint32_t>(RADIX - 1) << shift;
  }
  p.key = prefix;
  return p;
}

// Cluster fallback for a crossing bucket of more than CAP elements: radix
// passes over the keys of bucket `vb`, each a cluster-wide histogram
// (alternating buffers, so that a CTA never clears a histogram another may
// still be reading: two cluster barriers separate a read from the next clear).
__device__ __forceinline__ Pick cluster_select(int vb, Pick p, unsigned long long target, const uint32_t* key,
                                               float temperature, float mt, Shared& s, cg::cluster_group& cluster,
                                               int ncta, int& flip) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0, pmask = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const int buf = flip;
    flip ^= 1;
    for (int i = tid; i < NCOPY * RADIX; i += THREADS) {
      (&s.pm[0][0])[i] = 0;
      (&s.pc[0][0])[i] = 0;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const bool match = key[i] != kNoKey && (key[i] & pmask) == prefix && vbucket(key[i], temperature, mt) == vb;
      const unsigned long long q = match ? mass_of(key[i], temperature, mt) : 0ull;
      hist_add(q != 0, (key[i] >> shift) & (RADIX - 1), q, s.pm[(tid >> 5) % NCOPY], s.pc[(tid >> 5) % NCOPY]);
    }
    __syncthreads();
    if (tid < RADIX) {
      unsigned long long m = 0;
      unsigned c = 0;
#pragma unroll
      for (int k = 0; k < NCOPY; ++k) {
        m += s.pm[k][tid];
        c += s.pc[k][tid];
      }
      s.hmass[buf][tid] = m;
      s.hcount[buf][tid] = c;
    }
    cluster.sync();  // every CTA's histogram complete and visible
    unsigned long long m = 0, em, om;
    unsigned c = 0, en, on;
    if (tid < RADIX) {
      const int d = RADIX - 1 - tid;
#pragma unroll
      for (int r = 0; r < MAX_CTAS; ++r) {  // all remote loads in flight at once
        if (r < ncta) {
          m += cluster.map_shared_rank(&s.hmass[buf][0], r)[d];
          c += cluster.map_shared_rank(&s.hcount[buf][0], r)[d];
        }
      }
    }
    const int first = scan_cross(m, c, RADIX, p.above, target, s, em, en, om, on);
    p.above += em;
    p.n_above += en;
    p.ties = on;
    p.tie_mass = om;
    prefix |= static_cast<uint32_t>(RADIX - 1 - first) << shift;
    pmask |= static_cast<uint32_t>(RADIX - 1) << shift;
  }
  p.key = prefix;
  return p;
}

// The element (key) at which the descending running mass first exceeds
// `target` (< total mass). s.vmass / s.vcount hold the cluster's value-bucket
// totals; `sel` (0, 1) picks this call's candidate list, so that the two
// calls of a row never overwrite a list another CTA may still be reading.
__device__ __forceinline__ Pick select(unsigned long long target, int sel, const uint32_t* key, float temperature,
                                       float mt, Shared& s, cg::cluster_group& cluster, int ncta, int& flip) {
  const int tid = threadIdx.x;
  unsigned long long em, om;
  unsigned en, on;
  const int vb = scan_cross(s.vmass[tid], s.vcount[tid], VB, 0ull, target, s, em, en, om, on);
  Pick p{0, em, en, 0, 0};
  if (on <= static_cast<unsigned>(CAP)) {  // uniform: every CTA computed the same totals
    // gather this CTA's keys of bucket vb, then every CTA merges all lists
    if (tid == 0) s.cand_n[sel] = 0;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      if (key[i] != kNoKey && mass_of(key[i], temperature, mt) != 0 && vbucket(key[i], temperature, mt) == vb) {
        const unsigned slot = atomicAdd(&s.cand_n[sel], 1u);
        if (slot < static_cast<unsigned>(CAP)) s.cand[sel][slot] = key[i];
      }
    }
    cluster.sync();
    unsigned cnt[MAX_CTAS];
    int total = 0;
#pragma unroll
    for (int r = 0; r < MAX_CTAS; ++r) {
      cnt[r] = r < ncta ? *cluster.map_shared_rank(&s.cand_n[sel], r) : 0u;
      if (cnt[r] > static_cast<unsigned>(CAP)) cnt[r] = CAP;
      total += static_cast<int>(cnt[r]);
    }
    if (total > CAP) total = CAP;  // cannot happen: the bucket holds `on` <= CAP keys
    for (int i = tid; i < total; i += THREADS) {
      int r = 0, off = i;
      while (r < MAX_CTAS - 1 && off >= static_cast<int>(cnt[r])) off -= static_cast<int>(cnt[r++]);
      s.merged[i] = cluster.map_shared_rank(&s.cand[sel][0], r)[off];
    }
    __syncthreads();
    const Pick q = local_select(total, target - p.above, temperature, mt, s);
    p.key = q.key;
    p.above += q.above;
    p.n_above += q.n_above;
    p.ties = q.ties;
    p.tie_mass = q.tie_mass;
  } else {
    p = cluster_select(vb, p, target, key, temperature, mt, s, cluster, ncta, flip);
  }
  return p;
}

__global__ void __launch_bounds__(THREADS, 1)
top_p_kernel(const float* __restrict__ logits, int V, long long ld, float temperature, float top_p,
             const float* __restrict__ uniforms, long long* __restrict__ tokens, int* __restrict__ nucleus) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Shared& s = *reinterpret_cast<Shared*>(smem_raw);
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
#pragma unroll
  for (int r = 0; r < MAX_CTAS; ++r) {
    if (r < ncta) {
      const unsigned long long c = *cluster.map_shared_rank(&s.cta_max, r);
      gbest = c > gbest ? c : gbest;
    }
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

  // 2. integer masses, their total Q, and the value-bucket histogram
  const float mt = __fdiv_rn(m, temperature);
  for (int i = tid; i < VCOPY * VB; i += THREADS) {
    (&s.vpm[0][0])[i] = 0;
    (&s.vpc[0][0])[i] = 0;
  }
  __syncthreads();
  unsigned long long qsum = 0;
  {
    unsigned long long* vpm = s.vpm[(tid >> 5) % VCOPY];
    unsigned* vpc = s.vpc[(tid >> 5) % VCOPY];
    // Buckets are spread for real or random logits: plain atomics, except for
    // a warp whose lanes all fall into one bucket (rows of equal logits),
    // which adds once.
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const unsigned long long q = mass_of(key[i], temperature, mt);
      qsum += q;
      const bool has = q != 0;
      const int b = has ? vbucket(key[i], temperature, mt) : 0;
      const unsigned act = __ballot_sync(0xffffffffu, has);
      if (act && warp_uniform(act, has, static_cast<uint32_t>(b))) {
        if (has) {
          const unsigned long long sum = group_sum(act, q);
          if ((tid & 31) == __ffs(act) - 1) {
            atomicAdd(&vpm[b], sum);
            atomicAdd(&vpc[b], static_cast<unsigned>(__popc(act)));
          }
        }
      } else if (has) {
        atomicAdd(&vpm[b], q);
        atomicAdd(&vpc[b], 1u);
      }
    }
  }
  qsum = block_reduce<false>(qsum, s.warp64);  // (its barriers also complete the histogram copies)
  if (tid == 0) s.cta_mass = qsum;
  {
    unsigned long long vm = 0;
    unsigned vc = 0;
#pragma unroll
    for (int k = 0; k < VCOPY; ++k) {
      vm += s.vpm[k][tid];
      vc += s.vpc[k][tid];
    }
    s.vmass[tid] = vm;
    s.vcount[tid] = vc;
  }
  cluster.sync();
  unsigned long long Q = 0;
  {
    // cluster totals per bucket, kept in registers until no CTA reads this
    // CTA's own histogram any more (the next cluster barrier)
    unsigned long long vm = 0;
    unsigned vc = 0;
#pragma unroll
    for (int r = 0; r < MAX_CTAS; ++r) {
      if (r < ncta) {
        Q += *cluster.map_shared_rank(&s.cta_mass, r);
        vm += cluster.map_shared_rank(&s.vmass[0], r)[tid];
        vc += cluster.map_shared_rank(&s.vcount[0], r)[tid];
      }
    }
    cluster.sync();
    s.vmass[tid] = vm;
    s.vcount[tid] = vc;
    __syncthreads();
  }

  // 3. nucleus: keep a position iff the mass before it is <= top_p * Q
  int flip = 0;
  const unsigned long long tq =
      static_cast<unsigned long long>(floor(static_cast<double>(top_p) * static_cast<double>(Q)));
  unsigned long long kept_mass = Q;
  long long kept = V;
  if (Q > tq) {
    const Pick p = select(tq, 0, key, temperature, mt, s, cluster, ncta, flip);
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
  const Pick p2 = select(t2, 1, key, temperature, mt, s, cluster, ncta, flip);
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
#pragma unroll
  for (int r = 0; r < MAX_CTAS; ++r)
    if (r < rank) off += *cluster.map_shared_rank(&s.cta_ties, r);
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

int top_p_max_vocab() { return smp::MAX_CTAS * smp::CHUNK; }

cudaError_t launch_top_p(const float* logits, int rows, int V, long long ld, float temperature, float top_p,
                         const float* uniforms, long long* tokens, int* nucleus, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int ncta = (V + smp::CHUNK - 1) / smp::CHUNK;
  if (V <= 0 || ncta > smp::MAX_CTAS || rows > 65535) return cudaErrorInvalidValue;
  static bool attr[64] = {false};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr[dev]) {
    e = cudaFuncSetAttribute(smp::top_p_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(smp::Shared)));
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute cl[1];
  cl[0].id = cudaLaunchAttributeClusterDimension;
  cl[0].val.clusterDim.x = static_cast<unsigned>(ncta);
  cl[0].val.clusterDim.y = 1;
  cl[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(ncta), static_cast<unsigned>(rows), 1);
  cfg.blockDim = dim3(smp::THREADS, 1, 1);
  cfg.dynamicSmemBytes = sizeof(smp::Shared);
  cfg.stream = stream;
  cfg.attrs = cl;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, smp::top_p_kernel, logits, V, ld, temperature, top_p, uniforms, tokens, nucleus);
}

}  // namespace dsmoe
