/*
 * libdsmoe — B200-native (sm_100a) DeepSeek-R1 MoE block, C ABI.
 *
 * Drop-in boundary for the MoE hot path of sushruta/deepseek-on-one-gpu.
 * Every entry point below replaces one Python function of the reference
 * (cited as path:line inside that project). Arguments are raw device
 * pointers, sizes and a cudaStream_t; no framework types cross the ABI.
 *
 * Conventions
 *   - Every function returns 0 (DSMOE_OK) or a negative DSMOE_ERR_* code and
 *     never throws; dsmoe_last_error() returns a message for the calling
 *     thread's last failure.
 *   - All work is enqueued on `stream`; nothing blocks the host, nothing is
 *     allocated. Scratch memory comes from the caller ("workspace"), sized by
 *     the matching *_workspace_size() function.
 *   - Tensors are dense row-major: bf16 activations [tokens, hidden]; e4m3
 *     weights [out, in] with fp32 weight_scale_inv [out/128, in/128] that
 *     multiplies on dequantisation (the checkpoint format).
 *   - Expert groups: group 0 is the shared expert, group 1 + e is routed
 *     expert e. A weight bank holds n_slots experts; slot_of_expert maps each
 *     group to its slot.
 *   - Device errors (a bounded wait that timed out inside a kernel, a bad
 *     slot) are recorded in the workspace; dsmoe_read_status() fetches them.
 */
#ifndef DSMOE_H
#define DSMOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSMOE_API __attribute__((visibility("default")))
#else
#define DSMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* dsmoe_stream_t; /* == cudaStream_t */

enum {
  DSMOE_OK = 0,
  DSMOE_ERR_INVALID = -1,     /* bad argument (shape, pointer, alignment) */
  DSMOE_ERR_CUDA = -2,        /* a CUDA runtime/driver call failed */
  DSMOE_ERR_WORKSPACE = -3,   /* workspace too small */
  DSMOE_ERR_UNSUPPORTED = -4, /* shape or mode this build does not handle */
  DSMOE_ERR_DEVICE = -5       /* a kernel reported an error (see dsmoe_read_status) */
};

enum { DSMOE_ROUTER_REF = 0, DSMOE_ROUTER_V3 = 1 };

/* MoE fields of DeepSeekConfig (inference/config.py:32-52). */
typedef struct {
  int32_t hidden;          /* hidden_size, multiple of 128 */
  int32_t inter;           /* moe_intermediate_size, multiple of 128 */
  int32_t n_routed;        /* n_routed_experts = 32 * n_group */
  int32_t n_group;         /* <= 8 */
  int32_t topk_group;
  int32_t top_k;           /* num_experts_per_tok, <= 8 */
  int32_t router_mode;     /* DSMOE_ROUTER_REF or DSMOE_ROUTER_V3 */
  int32_t norm_topk_prob;
  float routed_scaling_factor;
} dsmoe_moe_config_t;

/* Device-resident expert weights of one MoE layer. */
typedef struct {
  const void* gate_weight;        /* bf16 [n_routed, hidden] */
  const float* score_bias;        /* fp32 [n_routed] (router v3) or NULL */
  int32_t n_slots;                /* experts held by the bank */
  const void* w_gate;             /* e4m3 [n_slots, inter, hidden] */
  const float* s_gate;            /* fp32 [n_slots, inter/128, hidden/128] */
  const void* w_up;               /* e4m3 [n_slots, inter, hidden] */
  const float* s_up;              /* fp32 [n_slots, inter/128, hidden/128] */
  const void* w_down;             /* e4m3 [n_slots, hidden, inter] */
  const float* s_down;            /* fp32 [n_slots, hidden/128, inter/128] */
  const int32_t* slot_of_expert;  /* device int32 [n_routed + 1]: group -> slot */
} dsmoe_layer_weights_t;

DSMOE_API const char* dsmoe_last_error(void);
DSMOE_API int dsmoe_version(void);

/* Scratch bytes for dsmoe_route / dsmoe_moe_forward / dsmoe_moe_experts at `tokens`. */
DSMOE_API size_t dsmoe_workspace_size(const dsmoe_moe_config_t* cfg, int32_t tokens);

/*
 * Router. Replaces route() (inference/ops.py:209-257) for router_mode REF;
 * REF ignores `score_bias` and applies no scaling factor (the reference
 * scales after the combine, inference/forward.py:153). V3 selects on
 * sigmoid + bias with top-2-sum group scores and returns weights already
 * multiplied by routed_scaling_factor.
 *   hidden [tokens, hidden] bf16 -> topk_idx [tokens, top_k] int64 (descending
 *   score), topk_w [tokens, top_k] fp32.
 */
DSMOE_API int dsmoe_route(const dsmoe_moe_config_t* cfg, const void* hidden, const void* gate_weight,
                const float* score_bias, int32_t tokens, int64_t* topk_idx, float* topk_w, void* workspace,
                size_t workspace_bytes, dsmoe_stream_t stream);

/*
 * Full MoE block. Replaces moe_block() (inference/forward.py:112-153):
 * route -> permute -> grouped FP8 gate/up (+SiLU*mul) -> grouped FP8 down ->
 * weighted combine with the shared expert. Every routed expert the routing
 * selects and the shared expert must be resident in `w` (slot_of_expert).
 *   hidden [tokens, hidden] bf16 -> out [tokens, hidden] bf16.
 * topk_idx / topk_w (optional, may be NULL) receive the routing as dsmoe_route.
 */
DSMOE_API int dsmoe_moe_forward(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden,
                      int32_t tokens, void* out, int64_t* topk_idx, float* topk_w, void* workspace,
                      size_t workspace_bytes, dsmoe_stream_t stream);

/*
 * Second half of dsmoe_moe_forward, for callers that route first and make the
 * selected experts resident afterwards (the expert-streaming path of
 * GPUTransfer.transfer_experts, inference/gpu_transfer.py:50-89): consumes the
 * routing that the preceding dsmoe_route left in the same workspace.
 */
DSMOE_API int dsmoe_moe_experts(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden,
                      int32_t tokens, void* out, void* workspace, size_t workspace_bytes, dsmoe_stream_t stream);

/* Scratch bytes for dsmoe_expert_ffn / dsmoe_fp8_linear. */
DSMOE_API size_t dsmoe_expert_ffn_workspace_size(int32_t tokens, int32_t hidden, int32_t inter);
DSMOE_API size_t dsmoe_fp8_linear_workspace_size(int32_t tokens, int32_t in_features, int32_t out_features);

/*
 * One expert FFN. Replaces expert_ffn() / swiglu() / dense_ffn()
 * (inference/ops.py:186-206): down(silu(gate(x)) * up(x)).
 * x [tokens, hidden] bf16 -> out [tokens, hidden] bf16; hidden and inter are
 * multiples of 128 up to 32768 (the dense layers 0-2 use inter = 18432).
 */
DSMOE_API int dsmoe_expert_ffn(const void* x, int32_t tokens, int32_t hidden, int32_t inter, const void* w_gate,
                     const float* s_gate, const void* w_up, const float* s_up, const void* w_down,
                     const float* s_down, void* out, void* workspace, size_t workspace_bytes,
                     dsmoe_stream_t stream);

/*
 * FP8 block-quantised linear. Replaces fp8_linear() (inference/ops.py:15-44)
 * for in/out features that are multiples of 128, up to 32768:
 *   out[t, o] = bf16( sum_i x[t, i] * weight[o, i] * scale_inv[o/128, i/128] ).
 */
DSMOE_API int dsmoe_fp8_linear(const void* x, int32_t tokens, int32_t in_features, int32_t out_features,
                     const void* weight, const float* scale_inv, void* out, void* workspace,
                     size_t workspace_bytes, dsmoe_stream_t stream);

/*
 * Measurement hook (no reference counterpart; the reference has no profiler
 * hooks). Registers up to 8 cudaEvent_t handles that the calling thread's
 * later dsmoe_moe_forward / dsmoe_moe_experts calls record on their stream at
 * stage boundaries: [0] before the router, [1] after it, [2] after the
 * permute, [3] after the gate/up GEMM, [4] after the SwiGLU/hi-lo split,
 * [5] after the down GEMM, [6] after the combine. n = 0 switches it off.
 */
DSMOE_API int dsmoe_set_profile_events(void* const* events, int32_t n);

/*
 * Measurement hook (no reference counterpart): enqueues on `stream` a probe in
 * which every SM writes its cycle counter and the global nanosecond timer to
 * out[2*smid] and out[2*smid+1] (device memory, n_slots pairs, n_slots >= the
 * SM count). Two probes around a timed region give each SM's mean clock over
 * it: (cycles after - before) / (ns after - before).
 */
DSMOE_API int dsmoe_clock_probe(uint64_t* out, int32_t n_slots, dsmoe_stream_t stream);

/*
 * RMSNorm, replaces `rms_norm` (inference/ops.py:10-13):
 *   out = bf16( bf16(x * 1/sqrt(mean(x^2) + eps)) * weight )
 * x, out [tokens][hidden] bf16, weight [hidden] bf16, hidden % 8 == 0, all
 * 16-byte aligned. The row mean is summed in a different order from torch's
 * CPU reduction, so 1/sqrt may differ from the reference in its last bit.
 */
DSMOE_API int dsmoe_rms_norm(const void* x, const void* weight, float eps, int32_t tokens, int32_t hidden,
                             void* out, dsmoe_stream_t stream);

/*
 * The FFN half of a MoE transformer layer, replaces
 * inference/forward.py:97-109 for layers >= first_k_dense_replace:
 *   out = hidden + moe_block(rms_norm(hidden, norm_weight, eps))
 * (bf16 residual add fused into the combine). `norm_weight` is the layer's
 * post_attention_layernorm weight [hidden] bf16; other arguments as for
 * dsmoe_moe_forward; the workspace is dsmoe_moe_layer_ffn_workspace_size
 * bytes (dsmoe_workspace_size plus the normalised activations). `out` must
 * not alias `hidden`.
 */
DSMOE_API size_t dsmoe_moe_layer_ffn_workspace_size(const dsmoe_moe_config_t* cfg, int32_t tokens);
DSMOE_API int dsmoe_moe_layer_ffn(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* weights,
                                  const void* hidden, const void* norm_weight, float eps, int32_t tokens, void* out,
                                  int64_t* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                                  dsmoe_stream_t stream);

/*
 * Host-side expert loader, replaces the disk read of
 * WeightStore._load_expert_from_disk (inference/weight_store.py:151-180):
 * copies n byte ranges (paths[i], offsets[i], sizes[i]) of safetensors shard
 * files into host buffers dsts[i] (pinned, typically one packed buffer per
 * expert) with pread on `threads` threads (1..64), ranges cut into 8 MiB
 * pieces. No GPU work. Returns DSMOE_ERR_INVALID for a missing file or a
 * range past its end.
 */
DSMOE_API int dsmoe_read_ranges(int32_t n, const char* const* paths, const uint64_t* offsets, const uint64_t* sizes,
                                void* const* dsts, int32_t threads);

/*
 * Overlap hook (no reference counterpart; the reference has no collectives).
 * Caps the persistent grid of the calling thread's later grouped-GEMM
 * launches at max_ctas CTAs (one per SM), leaving the other SMs free for a
 * collective running concurrently on another stream (the expert-parallel
 * all-to-all). 0 (the default) uses every SM. Results do not depend on it.
 */
DSMOE_API int dsmoe_set_gemm_sm_limit(int32_t max_ctas);

/*
 * Expert parallelism over W ranks (no counterpart in the reference, which is
 * single-GPU). Rank d owns routed experts
 * [d * experts_per_rank, (d+1) * experts_per_rank); gate and shared expert are
 * replicated. One layer step on every rank:
 *   1. dsmoe_route on the rank's tokens.
 *   2. dsmoe_ep_dispatch: one send row per (token, owning rank) - a token goes
 *      once to each rank that owns any of its experts - grouped by destination
 *      rank, inside a rank by token id. Writes send_counts[world] (device),
 *      tok_rows[tokens][world] (send row of each token's copy for each rank,
 *      -1 if none), send_tok[rows], send_idx[rows][top_k] (the token's experts
 *      on that rank as local ids in top-k order, -1 elsewhere), send_w (their
 *      routing weights) and send_hidden[rows][hidden] (bf16 copies).
 *      Capacity: tokens * min(top_k, world) rows.
 *   3. The caller exchanges counts and rows (all-to-all).
 *   4. dsmoe_moe_local on the received rows with the rank's experts (slot
 *      table over 1 + experts_per_rank groups; group 0 unused): one bf16
 *      partial row per received row, sum over its experts in top-k order.
 *   5. The caller returns the partial rows (all-to-all back, same splits).
 *   6. dsmoe_ep_combine: out[t] = bf16(shared[t] + bf16(scale * sum)), the sum
 *      over the returned rows of token t in rank order (bf16), shared[t] the
 *      shared expert on the rank's own tokens (dsmoe_expert_ffn).
 */
DSMOE_API int dsmoe_ep_dispatch(const int64_t* topk_idx, const float* topk_w, const void* hidden, int32_t tokens,
                                int32_t top_k, int32_t hidden_size, int32_t world, int32_t experts_per_rank,
                                int32_t* send_counts, int32_t* tok_rows, int32_t* send_tok, int32_t* send_idx,
                                float* send_w, void* send_hidden, dsmoe_stream_t stream);
DSMOE_API size_t dsmoe_moe_local_workspace_size(const dsmoe_moe_config_t* cfg_local, int32_t rows);
DSMOE_API int dsmoe_moe_local(const dsmoe_moe_config_t* cfg_local, const dsmoe_layer_weights_t* w, const void* hidden,
                              int32_t rows, const int32_t* local_idx, const float* local_w, void* partial_out,
                              void* workspace, size_t workspace_bytes, dsmoe_stream_t stream);
DSMOE_API int dsmoe_ep_combine(const void* partials, const int32_t* tok_rows, int32_t tokens, int32_t world,
                               int32_t hidden_size, const void* shared_out, float scale, void* out,
                               dsmoe_stream_t stream);

/*
 * Expert parallelism over peer memory (no counterpart in the reference; the
 * exchange without NCCL all-to-all). Every rank allocates, once, receive
 * buffers for world * cap rows (hidden rows and routing metadata, see
 * dsmoe_ep_meta_bytes) and a return buffer of world * cap partial rows, in
 * device memory that the other ranks map (dsmoe_ipc_alloc / dsmoe_ipc_open).
 * One step on rank `rank` (tokens <= cap):
 *   1. dsmoe_ep_plan: like dsmoe_ep_dispatch without the row copy (send
 *      counts, tok_rows, send_tok, send_idx, send_w).
 *   2. the caller gathers every rank's send_counts into counts_all
 *      [world][world] (row = sending rank) on every rank.
 *   3. dsmoe_ep_push: writes each send row straight into the destination
 *      rank's receive buffers (peer_recv_hidden[d], peer_recv_meta[d]: the
 *      buffers' addresses in this process) at row
 *      sum_{s < rank} counts_all[s][d] + k, with its local expert ids,
 *      weights and origin (rank, k); rewrites tok_rows[t][d] to d * cap + k.
 *   4. a barrier across ranks (the caller's), then on every rank
 *      dsmoe_moe_local_peer over its rows received (sum of counts_all[.][rank];
 *      given counts_all, the library counts them on the device and `rows` is
 *      only a bound, e.g. world * cap, so the host never reads the counts):
 *      the grouped GEMMs of dsmoe_moe_local, whose combine writes each partial
 *      row into the ORIGIN rank's return buffer (peer_return[s]) at row
 *      rank * cap + k.
 *   5. a barrier, then dsmoe_ep_combine over the own return buffer with the
 *      rewritten tok_rows.
 * Receive metadata layout (int32): local expert ids [world*cap][top_k],
 * weights as fp32 bits [world*cap][top_k], origin [world*cap][2].
 */
DSMOE_API int dsmoe_ep_plan(const int64_t* topk_idx, const float* topk_w, int32_t tokens, int32_t top_k, int32_t world,
                            int32_t experts_per_rank, int32_t* send_counts, int32_t* tok_rows, int32_t* send_tok,
                            int32_t* send_idx, float* send_w, dsmoe_stream_t stream);
DSMOE_API int dsmoe_ep_push(const void* hidden, int32_t tokens, int32_t top_k, int32_t hidden_size, int32_t world,
                            int32_t rank, int32_t cap, const int32_t* counts_all, const int32_t* send_tok,
                            const int32_t* send_idx, const float* send_w, int32_t* tok_rows,
                            const uint64_t* peer_recv_hidden, const uint64_t* peer_recv_meta, int32_t* device_status,
                            int32_t max_blocks, dsmoe_stream_t stream);
/* device_status (may be NULL): error word set (code 6) when the gathered
 * counts do not fit the receive buffers; such rows are not written and their
 * tok_rows entry becomes -1. max_blocks > 0 caps the push's grid, so that it
 * can run beside a grouped GEMM whose grid leaves that many SMs free
 * (dsmoe_set_gemm_sm_limit). */
DSMOE_API int dsmoe_moe_local_peer(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* weights,
                                   const void* recv_hidden, int32_t rows, const int32_t* recv_meta, int32_t world,
                                   int32_t rank, int32_t cap, const uint64_t* peer_return, const int32_t* counts_all,
                                   void* workspace, size_t workspace_bytes, dsmoe_stream_t stream);
DSMOE_API size_t dsmoe_ep_meta_bytes(int32_t world, int32_t cap, int32_t top_k);

/*
 * Device memory other processes on this node can map (CUDA IPC; used for
 * the peer-memory exchange buffers). dsmoe_ipc_alloc allocates `bytes` and
 * writes a DSMOE_IPC_HANDLE_BYTES handle; another process maps it with
 * dsmoe_ipc_open (not in the allocating process itself) and unmaps it with
 * dsmoe_ipc_close; the owner releases it with dsmoe_ipc_free. These allocate:
 * call them at set-up, not per step.
 */
#define DSMOE_IPC_HANDLE_BYTES 64
DSMOE_API int dsmoe_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
DSMOE_API int dsmoe_ipc_open(const void* handle, void** dev_ptr);
DSMOE_API int dsmoe_ipc_close(void* dev_ptr);
DSMOE_API int dsmoe_ipc_free(void* dev_ptr);

/*
 * Allocation-free variant of dsmoe_expert_ffn (no counterpart in the
 * reference; an addition of this library).
 *
 * Some callers cannot allocate device memory at call time: a runtime that
 * owns all device memory through its own fixed pool and forbids any other
 * allocation, code that runs while an allocator lock is held (for instance
 * from a memory-pressure or allocation callback), and latency-critical paths
 * that must not take an allocation that can block, synchronize the device or
 * fail under memory pressure. This entry point computes the same result as
 * dsmoe_expert_ffn without a workspace argument and without calling cudaMalloc,
 * cudaFree or any allocating routine: its scratch is a fixed array of
 * DSMOE_NOALLOC_SCRATCH_BYTES inside the library, one per GPU, held by every
 * GPU that loads the library until the process exits.
 *
 *   - The caller still provides x, the weights and out (same layouts as
 *     dsmoe_expert_ffn).
 *   - Shapes whose scratch need (dsmoe_expert_ffn_workspace_size) exceeds
 *     DSMOE_NOALLOC_SCRATCH_BYTES are rejected with DSMOE_ERR_WORKSPACE before
 *     any work is enqueued (about 300 tokens at hidden 7168, inter 2048).
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls on a device share the one array, and it keeps the previous
 *     call's contents (the call clears what must start at zero). Calls whose
 *     work can overlap on the GPU race on the array: issue them on one stream
 *     or order them with events.
 *   - A kernel failure (a bounded wait that ran out) is recorded in the
 *     array's error word, which stays set until dsmoe_read_status(NULL, ...)
 *     reads and clears it; rc 0 only means the work was enqueued.
 */
#define DSMOE_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
DSMOE_API int dsmoe_expert_ffn_noalloc(const void* x, int32_t tokens, int32_t hidden, int32_t inter,
                                       const void* w_gate, const float* s_gate, const void* w_up, const float* s_up,
                                       const void* w_down, const float* s_down, void* out, dsmoe_stream_t stream);

/*
 * Device-resident expert slot cache for streaming mode (replaces the host side
 * of GPUTransfer.transfer_experts, inference/gpu_transfer.py:50-89, whose
 * .tolist() and synchronize() (:60, :79) stop the host once per token and
 * layer). A layer's routed experts live in pinned host memory; the GPU keeps a
 * bank of n_slots expert slots (the dsmoe_layer_weights_t layout) and the
 * group -> slot table the grouped GEMMs read. dsmoe_slotcache_step, called
 * with the step's routing (the topk_idx of dsmoe_route) before
 * dsmoe_moe_experts, runs two kernels on `stream`:
 *   - plan: refresh the recency of the needed experts already in a slot and
 *     give each missing expert (in id order) the least recently used slot the
 *     step does not need (empty slots first, ties to the lowest slot, the
 *     shared expert's slot never), updating slot_of;
 *   - fill: copy the missing experts' six tensors from host memory (read by
 *     the SMs over the host link) into their slots.
 * No host read and no host wait; a step needing more experts than free slots
 * sets code 4 in *status.
 * state: dsmoe_slotcache_state_bytes(n_slots) bytes of int32, caller-owned:
 *   [0] step clock, [1] experts copied by the last step, [2] hits, [3] misses
 *   (cumulative), then group_in_slot[n_slots] (-1 empty, 0 the shared expert,
 *   1 + e routed expert e), last_use[n_slots] (-1 empty), and two copy lists
 *   of n_slots entries. Initialise clock/counters to 0 and group_in_slot /
 *   last_use to the bank's contents, with slot_of consistent with them.
 * host_src: device array [n_experts][6] of device-usable addresses of routed
 *   expert e's w_gate, s_gate, w_up, s_up, w_down, s_down in pinned host
 *   memory, produced by dsmoe_map_host_pointers from the host addresses.
 */
typedef struct {
  int32_t n_experts;  /* routed experts of the layer (<= 1023) */
  int32_t n_slots;    /* bank slots, the shared expert's included */
  int32_t hidden;     /* multiples of 128 */
  int32_t inter;
  void* w_gate;       /* bank tensors [n_slots][...], 16-byte aligned */
  float* s_gate;
  void* w_up;
  float* s_up;
  void* w_down;
  float* s_down;
  int32_t* slot_of;   /* [n_experts + 1] group -> slot, -1 absent */
  int32_t* state;
  const uint64_t* host_src;
  int32_t* status;    /* device error word */
} dsmoe_slotcache_t;
DSMOE_API size_t dsmoe_slotcache_state_bytes(int32_t n_slots);
DSMOE_API int dsmoe_slotcache_step(const dsmoe_slotcache_t* cache, const int64_t* topk_idx, int32_t n_pairs,
                                   dsmoe_stream_t stream);
/* Host addresses of pinned (page-locked, mapped) host memory -> the addresses
 * kernels use for it (cudaHostGetDevicePointer); entries must be 16-byte
 * aligned. Set-up call, host only. */
DSMOE_API int dsmoe_map_host_pointers(const uint64_t* host_ptrs, int32_t n, uint64_t* dev_ptrs);

/*
 * Next-token sampling, replaces `sample` (inference/engine.py:166-190) and
 * the .item() read of the decode loop (engine.py:116-117, 142-151): the token
 * ids stay on the device.
 *   logits    [rows][row_stride] fp32 (vocab used per row, 1 <= vocab <= 131072)
 *   temperature == 0: tokens[r] = first index of the row maximum (argmax);
 *   temperature > 0:  softmax(logits / temperature), keep the shortest
 *     descending prefix whose preceding mass stays <= top_p (the reference's
 *     mask `cumulative - p > top_p`), and take the element where the
 *     descending running mass of the kept set first exceeds
 *     uniforms[r] * (kept mass) (inverse CDF with a caller-drawn uniform in
 *     [0, 1); the reference draws it inside torch.multinomial).
 *   tokens        [rows] int64 output; -1 for a row whose maximum logit is not
 *                 finite (the reference's softmax is NaN there)
 *   nucleus_sizes [rows] int32 output (NULL allowed): kept elements per row
 * Equal logits are ordered by index. Masses are exact integers
 * (round(2^40 * exp(l/T - max/T))), so results are deterministic; they can
 * differ from the reference's fp32 cumsum where a boundary lies within
 * ~1e-6 of top_p or of the drawn uniform. One cluster of up to 8 CTAs per row.
 * rows <= 65535; temperature >= 0 and finite; top_p >= 0 (>= 1 keeps all);
 * uniforms may be NULL when temperature == 0.
 */
DSMOE_API int dsmoe_sample_top_p(const float* logits, int32_t rows, int32_t vocab, int64_t row_stride,
                                 float temperature, float top_p, const float* uniforms, int64_t* tokens,
                                 int32_t* nucleus_sizes, dsmoe_stream_t stream);

/* Reads (synchronously) and clears the device error word kept in `workspace`.
 * workspace == NULL reads the error word of dsmoe_expert_ffn_noalloc's
 * library-owned scratch on the current device: that entry point has no
 * workspace argument, and its error word stays set (first error wins) until
 * read here, so a failure is not lost to the next call. */
DSMOE_API int dsmoe_read_status(void* workspace, int32_t* device_status, dsmoe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DSMOE_H */
