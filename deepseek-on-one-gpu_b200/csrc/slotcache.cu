// Device-resident expert slot cache (streaming mode: a layer's routed experts
// live in pinned host memory, the GPU holds a bank of n_slots expert slots).
//
// Replaces the host side of GPUTransfer.transfer_experts
// (inference/gpu_transfer.py:50-89): the reference reads each token's expert
// ids back to the host (.tolist(), :60), copies that token's 8 experts into 8
// slots on a side stream and blocks the host on synchronize() (:79) before
// the expert FFNs. Here the routing never leaves the device; per step and
// layer, on the caller's stream before the expert GEMMs:
//   plan   one CTA: marks the expert groups the step's (token, k) pairs
//          need, refreshes the recency of those already in a slot, and gives
//          each missing expert (in expert-id order) the least recently used
//          slot that the step does not need (ties: lowest slot; empty slots
//          first; the shared expert's slot is never taken). It updates
//          slot_of / group_in_slot and writes the copy list.
//   fill   copies each listed expert's six tensors (three e4m3 weights and
//          their fp32 scales) from pinned host memory, read by the SMs over
//          the host link with 16-byte loads, into its slot.
// The grouped GEMMs then find every needed group through slot_of.
//
// State (int32, caller-owned, see dsmoe.h): [0] step clock, [1] copies of the
// last step, [2] hits, [3] misses (cumulative), then group_in_slot[n_slots],
// last_use[n_slots], copy_group[n_slots], copy_slot[n_slots].
#include <cstdio>

#include "../../include/dsmoe.h"
#include "common.cuh"
#include "kernels.h"

namespace dsmoe {

namespace sc {
constexpr int PLAN_THREADS = 512;
constexpr int MAX_GROUPS = 1024;
constexpr int PINNED = 0x7fffffff;

struct StateView {
  int* clock;
  int* n_copy;
  int* hits;
  int* misses;
  int* group_in_slot;
  int* last_use;
  int* copy_group;
  int* copy_slot;
};

__device__ __forceinline__ StateView view(int* st, int n_slots) {
  StateView v;
  v.clock = st;
  v.n_copy = st + 1;
  v.hits = st + 2;
  v.misses = st + 3;
  v.group_in_slot = st + 4;
  v.last_use = v.group_in_slot + n_slots;
  v.copy_group = v.last_use + n_slots;
  v.copy_slot = v.copy_group + n_slots;
  return v;
}

__global__ void __launch_bounds__(PLAN_THREADS) plan_kernel(const int64_t* __restrict__ idx, int n_pairs,
                                                            int n_experts, int n_slots, int* __restrict__ slot_of,
                                                            int* __restrict__ state, int* __restrict__ status) {
  __shared__ uint32_t need[MAX_GROUPS / 32];
  __shared__ int s_miss[MAX_GROUPS];
  __shared__ int s_nmiss, s_hits;
  __shared__ unsigned long long s_best[PLAN_THREADS / 32];
  StateView st = view(state, n_slots);
  const int tid = threadIdx.x;
  const int n_groups = n_experts + 1;
  for (int i = tid; i < MAX_GROUPS / 32; i += blockDim.x) need[i] = 0;
  if (tid == 0) {
    s_nmiss = 0;
    s_hits = 0;
  }
  __syncthreads();
  for (int p = tid; p < n_pairs; p += blockDim.x) {
    const int64_t e = idx[p];
    if (e >= 0 && e < n_experts) atomicOr(&need[(e + 1) >> 5], 1u << ((e + 1) & 31));
  }
  __syncthreads();
  const int clock = *st.clock + 1;
  // hits: refresh recency (group 0, the shared expert, is never routed)
  for (int g = 1 + tid; g < n_groups; g += blockDim.x) {
    if ((need[g >> 5] >> (g & 31)) & 1u) {
      const int s = slot_of[g];
      if (s >= 0) {
        st.last_use[s] = clock;
        atomicAdd(&s_hits, 1);
      }
    }
  }
  __syncthreads();
  // misses in expert-id order (one thread: at most n_experts checks)
  if (tid == 0) {
    int n = 0;
    for (int g = 1; g < n_groups; ++g)
      if (((need[g >> 5] >> (g & 31)) & 1u) && slot_of[g] < 0) s_miss[n++] = g;
    s_nmiss = n;
  }
  __syncthreads();
  const int nmiss = s_nmiss;
  int placed = 0;
  for (int m = 0; m < nmiss; ++m) {
    // least recently used slot not needed this step: key (last_use, slot),
    // empty slots (last_use -1) first, slots used or filled this step
    // (last_use == clock) and the shared expert's slot excluded
    unsigned long long best = ~0ull;
    for (int s = tid; s < n_slots; s += blockDim.x) {
      const int lu = st.last_use[s];
      if (lu == clock || lu == PINNED || st.group_in_slot[s] == 0) continue;
      const unsigned long long key =
          (static_cast<unsigned long long>(static_cast<unsigned int>(lu + 1)) << 32) | static_cast<unsigned int>(s);
      best = key < best ? key : best;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other < best ? other : best;
    }
    if ((tid & 31) == 0) s_best[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long b = s_best[0];
      for (int w = 1; w < PLAN_THREADS / 32; ++w) b = s_best[w] < b ? s_best[w] : b;
      if (b == ~0ull) {
        atomicCAS(status, 0, kDevBadSlot);  // more experts needed than slots
      } else {
        const int v = static_cast<int>(b & 0xffffffffu);
        const int g = s_miss[m];
        const int old = st.group_in_slot[v];
        if (old > 0) slot_of[old] = -1;
        slot_of[g] = v;
        st.group_in_slot[v] = g;
        st.last_use[v] = clock;
        st.copy_group[placed] = g;
        st.copy_slot[placed] = v;
        ++placed;
      }
    }
    __syncthreads();
    if (tid == 0) s_nmiss = placed;  // placed so far (broadcast for the next miss)
    __syncthreads();
    placed = s_nmiss;
  }
  if (tid == 0) {
    *st.clock = clock;
    *st.n_copy = placed;
    *st.hits += s_hits;
    *st.misses += nmiss;
  }
}

// Copy the listed experts' tensors from host memory into their slots.
// src[(e * 6) + t]: device-usable address of tensor t (w_gate, s_gate, w_up,
// s_up, w_down, s_down) of routed expert e; dst[t] the bank tensor base,
// bytes[t] its per-slot size (a multiple of 16).
struct FillArgs {
  const uint64_t* src;
  uint64_t dst[6];
  uint64_t bytes[6];
};

__global__ void __launch_bounds__(256) fill_kernel(FillArgs a, const int* __restrict__ state, int n_slots) {
  const int* n_copy = state + 1;
  const int* copy_group = state + 4 + 2 * n_slots;
  const int* copy_slot = copy_group + n_slots;
  const int n = *n_copy;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (int i = 0; i < n; ++i) {
    const int e = copy_group[i] - 1;
    const int s = copy_slot[i];
#pragma unroll 1
    for (int t = 0; t < 6; ++t) {
      const uint4* src = reinterpret_cast<const uint4*>(a.src[static_cast<size_t>(e) * 6 + t]);
      uint4* dst = reinterpret_cast<uint4*>(a.dst[t] + static_cast<uint64_t>(s) * a.bytes[t]);
      const size_t n16 = a.bytes[t] / 16;
      size_t j = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
      // four independent 16-byte loads in flight per thread: host-link reads
      // have a long latency
      for (; j + 3 * stride < n16; j += 4 * stride) {
        const uint4 v0 = src[j], v1 = src[j + stride], v2 = src[j + 2 * stride], v3 = src[j + 3 * stride];
        dst[j] = v0;
        dst[j + stride] = v1;
        dst[j + 2 * stride] = v2;
        dst[j + 3 * stride] = v3;
      }
      for (; j < n16; j += stride) dst[j] = src[j];
    }
  }
}
}  // namespace sc

}  // namespace dsmoe

using namespace dsmoe;

extern "C" {

size_t dsmoe_slotcache_state_bytes(int32_t n_slots) {
  if (n_slots < 1) return 0;
  return sizeof(int32_t) * (4 + 4 * static_cast<size_t>(n_slots));
}

int dsmoe_map_host_pointers(const uint64_t* host_ptrs, int32_t n, uint64_t* dev_ptrs) {
  if (n < 0 || (n > 0 && (!host_ptrs || !dev_ptrs))) return set_last_error(DSMOE_ERR_INVALID, "bad arguments");
  for (int i = 0; i < n; ++i) {
    if (host_ptrs[i] % 16) return set_last_error(DSMOE_ERR_INVALID, "host tensor not 16-byte aligned");
    void* d = nullptr;
    const cudaError_t e = cudaHostGetDevicePointer(&d, reinterpret_cast<void*>(host_ptrs[i]), 0);
    if (e != cudaSuccess || !d) {
      char buf[160];
      snprintf(buf, sizeof(buf), "cudaHostGetDevicePointer(entry %d): %s (not pinned host memory?)", i,
               cudaGetErrorString(e));
      return set_last_error(DSMOE_ERR_CUDA, buf);
    }
    dev_ptrs[i] = reinterpret_cast<uint64_t>(d);
  }
  return DSMOE_OK;
}

int dsmoe_slotcache_step(const dsmoe_slotcache_t* c, const int64_t* topk_idx, int32_t n_pairs,
                         dsmoe_stream_t stream) {
  if (!c) return set_last_error(DSMOE_ERR_INVALID, "slot cache is NULL");
  if (c->n_experts < 1 || c->n_experts + 1 > sc::MAX_GROUPS || c->n_slots < 2 || c->hidden <= 0 ||
      c->hidden % 128 || c->inter <= 0 || c->inter % 128 || n_pairs < 0)
    return set_last_error(DSMOE_ERR_INVALID, "slot cache: bad sizes");
  const void* ps[10] = {c->w_gate, c->s_gate, c->w_up, c->s_up, c->w_down, c->s_down, c->slot_of, c->state,
                        c->host_src, c->status};
  for (const void* p : ps)
    if (!p) return set_last_error(DSMOE_ERR_INVALID, "slot cache: NULL pointer");
  if (n_pairs > 0 && !topk_idx) return set_last_error(DSMOE_ERR_INVALID, "topk_idx is NULL");
  for (int t = 0; t < 6; ++t)
    if (reinterpret_cast<uintptr_t>(ps[t]) % 16) return set_last_error(DSMOE_ERR_INVALID, "bank not 16-byte aligned");
  const uint64_t fh = static_cast<uint64_t>(c->inter) * c->hidden;
  const uint64_t sfh = static_cast<uint64_t>(c->inter / 128) * (c->hidden / 128) * sizeof(float);
  if (sfh % 16) return set_last_error(DSMOE_ERR_UNSUPPORTED, "slot cache: scale blocks not a multiple of 16 bytes");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  sc::plan_kernel<<<1, sc::PLAN_THREADS, 0, s>>>(topk_idx, n_pairs, c->n_experts, c->n_slots, c->slot_of,
                                                 c->state, c->status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(DSMOE_ERR_CUDA, cudaGetErrorString(e));
  sc::FillArgs a;
  a.src = c->host_src;
  const void* dst[6] = {c->w_gate, c->s_gate, c->w_up, c->s_up, c->w_down, c->s_down};
  for (int t = 0; t < 6; ++t) {
    a.dst[t] = reinterpret_cast<uint64_t>(dst[t]);
    a.bytes[t] = (t & 1) ? sfh : fh;
  }
  int dev = 0, n_sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
  sc::fill_kernel<<<2 * n_sm, 256, 0, s>>>(a, c->state, c->n_slots);
  e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(DSMOE_ERR_CUDA, cudaGetErrorString(e));
  return DSMOE_OK;
}

}  // extern "C"
