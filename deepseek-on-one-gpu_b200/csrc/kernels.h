// Internal launch interface between the C ABI (api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsmoe {

// Records `msg` as the calling thread's dsmoe_last_error() and returns `code`.
int set_last_error(int code, const char* msg);
// Device address of the current device's allocation-free scratch status word
// (noalloc.cu); nullptr with the reason in *err on failure.
void* noalloc_status_word(const char** err);

// Group-table convention used by every kernel: group 0 is the shared expert
// (every token, in token order), group 1 + e is routed expert e.
struct GemmParams {
  const int32_t* counts;      // [n_groups] tokens per group
  const int32_t* row_start;   // [n_groups] first permuted row (multiple of 32)
  const int32_t* unit_start;  // [n_groups + 1] prefix sum of work units
  const int32_t* slot_of;     // [n_groups] weight-bank slot of each group
  const float* wscale0;       // [n_slots][M/128][K/128] scales of weight matrix 0
  const float* wscale1;       // same for matrix 1 (n_mat == 2)
  int n_groups;
  int n_slots;
  int n_mat;  // weight matrices per launch: 2 = gate and up, 1 = down / single linear
  int M;      // rows of one weight matrix per expert (output features)
  int K;      // reduction length
  int P;      // rows of one activation half (hi rows [0,P), lo rows [P,2P))
  const float* sx;      // [P] per-row activation scale
  __nv_bfloat16* y;     // output: bf16 [P][n_mat * M]
  int* status;          // device error word
};

// Token tile (max tokens per work unit) of the grouped GEMM for a launch over
// `tokens` tokens; the unit plan (permute.cu) must count tiles of this size.
int gemm_tile_tokens(int tokens);
// x: activation map with `tile`-row boxes, x32: the same rows with 32-row boxes.
cudaError_t launch_grouped_gemm(const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
                                const CUtensorMap& x32, const GemmParams& p, int tile, int grid, cudaStream_t stream);

// Clock probe (clockprobe.cu): out[2*smid] = SM cycle counter, out[2*smid+1] =
// global ns timer, for every SM a block lands on (smid < n_slots).
cudaError_t launch_clock_probe(unsigned long long* out, int n_slots, int n_sm, cudaStream_t stream);

// SwiGLU + hi/lo split (swiglu_quant.cu)
// rows of real (token, group) pairs only: row_start[n_groups + 1], counts[n_groups]
cudaError_t launch_swiglu_quant(const __nv_bfloat16* gu, int F, const int32_t* row_start, const int32_t* counts,
                                int n_groups, int P, uint8_t* hq, float* hs, cudaStream_t stream);

// Router (router_tc.cu logits, router.cu selection)
int router_tc_ksplit(int T, int H, int num_sms);
cudaError_t launch_router_logits_tc(const CUtensorMap& tm_x, const CUtensorMap& tm_g, float* partial, int T, int H,
                                    int E, int ksplit, int* status, cudaStream_t stream);
cudaError_t launch_router_select(const float* partial, int ksplit, const float* bias, int T, int E, int n_group,
                                 int topk_group, int top_k, int mode, int norm, float scaling, int32_t* idx,
                                 int64_t* idx64, float* w, cudaStream_t stream);

// Permutation (permute.cu)
// n_rows (optional): a row count held on the device; work past it is skipped
// (n_pairs / T are then bounds that size the grids).
cudaError_t launch_count(const int32_t* idx, int n_pairs, int32_t* counts, int n_groups, cudaStream_t stream,
                         const int32_t* n_rows = nullptr, int per_row = 1);
cudaError_t launch_plan(int32_t* counts, int n_groups, int shared_tokens, int tile, int mt_up, int mt_dn,
                        int32_t* row_start, int32_t* cursor, int32_t* ustart_up, int32_t* ustart_dn,
                        cudaStream_t stream);
cudaError_t launch_quant_scatter(const void* x, int T, int H, const int32_t* idx, int top_k, int n_groups,
                                 int has_shared, const int32_t* row_start, int32_t* cursor, int P, uint8_t* xq,
                                 float* sx, int32_t* pos, cudaStream_t stream, const int32_t* n_rows = nullptr);

// Combine (combine.cu)
// residual (optional, [T][H]): out = bf16(residual + combined row)
// peer_out (optional): row t goes to peer_out[origin[2t]] + (me * cap + origin[2t+1]) * H instead of out + t * H
cudaError_t launch_combine(const __nv_bfloat16* y, int T, int H, const int32_t* pos, const float* w, int top_k,
                           const int32_t* row_start, float scale, int has_shared, const __nv_bfloat16* residual,
                           __nv_bfloat16* out, cudaStream_t stream, const int32_t* origin = nullptr,
                           const uint64_t* peer_out = nullptr, int me = 0, int cap = 0,
                           const int32_t* n_rows = nullptr);

// y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * w), one row of H per token
cudaError_t launch_rmsnorm(const void* x, const void* w, float eps, int T, int H, void* y, cudaStream_t stream);

// Temperature + top-p sampling (sampler.cu), one cluster per row
int top_p_max_vocab();
cudaError_t launch_top_p(const float* logits, int rows, int V, long long ld, float temperature, float top_p,
                         const float* uniforms, long long* tokens, int* nucleus, cudaStream_t stream);

// Expert parallelism (ep.cu)
cudaError_t launch_ep_dispatch(const int64_t* idx, const float* w, const void* x, int T, int K, int H, int W, int El,
                               int32_t* counts, int32_t* tok_rows, int32_t* send_tok, int32_t* send_idx,
                               float* send_w, void* send_x, cudaStream_t stream);
cudaError_t launch_ep_plan(const int64_t* idx, const float* w, int T, int K, int W, int El, int32_t* counts,
                           int32_t* tok_rows, int32_t* send_tok, int32_t* send_idx, float* send_w, cudaStream_t stream);
// status (optional): device error word for rows whose counts do not fit the
// receive buffers; max_blocks > 0 caps the grid (SMs left to concurrent work).
cudaError_t launch_ep_push(const void* x, int T, int H, int K, int W, int me, int cap, const int32_t* counts_all,
                           const int32_t* send_tok, const int32_t* send_idx, const float* send_w, int32_t* tok_rows,
                           const uint64_t* recv_x, const uint64_t* recv_meta, int* status, int max_blocks,
                           cudaStream_t stream);
// *out = sum over s of counts_all[s][me]
cudaError_t launch_ep_recv_rows(const int32_t* counts_all, int W, int me, int32_t* out, cudaStream_t stream);
cudaError_t launch_ep_combine(const void* part, const int32_t* tok_rows, int T, int W, int H, const void* shared,
                              float scale, void* out, cudaStream_t stream);

}  // namespace dsmoe
