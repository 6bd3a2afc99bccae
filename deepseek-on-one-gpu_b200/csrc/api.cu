// libdsmoe C ABI: argument checks, workspace planning, TMA descriptors and
// the launch sequence of the MoE block. See include/dsmoe.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/dsmoe.h"
#include "kernels.h"

namespace dsmoe {
namespace {

thread_local std::string g_err;

// Optional stage-boundary events (dsmoe_set_profile_events), per host thread.
constexpr int kMaxProf = 8;
thread_local cudaEvent_t g_prof[kMaxProf] = {};
thread_local int g_nprof = 0;

void prof(int i, cudaStream_t s) {
  if (i < g_nprof && g_prof[i]) cudaEventRecord(g_prof[i], s);
}

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define DSMOE_CUDA(call)                                                                              \
  do {                                                                                                \
    cudaError_t e_ = (call);                                                                          \
    if (e_ != cudaSuccess) return fail(DSMOE_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                           \
  } while (0)

constexpr size_t kAlign = 256;
size_t align_up(size_t v, size_t a = kAlign) { return (v + a - 1) / a * a; }
int round32(int v) { return (v + 31) & ~31; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ------------------------------------------------------------------ TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major map: `rows` x `cols` elements, box `box_rows` x `box_cols`.
int make_map(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t cols, uint64_t rows,
             uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(DSMOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DSMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d): rows=%llu cols=%llu box=%ux%u", int(r),
                (unsigned long long)rows, (unsigned long long)cols, box_rows, box_cols);
  return DSMOE_OK;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// --------------------------------------------------------------- workspace
struct Ws {
  size_t status = 0, counts = 0, cursor = 0, row_start = 0, us_up = 0, us_dn = 0, slot0 = 0;
  size_t partial = 0, idx = 0, w = 0, pos = 0, xq = 0, sx = 0, hq = 0, hs = 0, y = 0, total = 0;
  int P = 0, ksplit = 1, NG = 1;
};

// Routed MoE block: groups = shared + n_routed; rows = shared segment +
// routed segments, every segment padded to a multiple of 32 rows.
Ws plan_moe(int T, int H, int F, int E, int K) {
  Ws w;
  w.NG = E + 1;
  const long long pairs = static_cast<long long>(T) * K;
  const long long pad = 31LL * (pairs < E ? pairs : E);
  w.P = round32(T) + round32(static_cast<int>(pairs + pad));
  w.ksplit = router_ksplit(T, H, E, 148);
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes); return at; };
  w.status = take(sizeof(int));
  w.counts = take(4 * w.NG);
  w.cursor = take(4 * w.NG);
  w.row_start = take(4 * (w.NG + 1));
  w.us_up = take(4 * (w.NG + 1));
  w.us_dn = take(4 * (w.NG + 1));
  w.slot0 = take(4);
  w.partial = take(sizeof(float) * static_cast<size_t>(w.ksplit) * T * E);
  w.idx = take(4 * static_cast<size_t>(pairs));
  w.w = take(4 * static_cast<size_t>(pairs));
  w.pos = take(4 * static_cast<size_t>(pairs));
  w.xq = take(2 * static_cast<size_t>(w.P) * H);
  w.sx = take(4 * static_cast<size_t>(H / 128) * w.P);
  w.hq = take(2 * static_cast<size_t>(w.P) * F);
  w.hs = take(4 * static_cast<size_t>(F / 128) * w.P);
  w.y = take(2 * static_cast<size_t>(w.P) * H);
  w.total = o;
  return w;
}

// Single expert (or single linear): one group holding every token in order.
Ws plan_single(int T, int K_in, int F /* 0 for a plain linear */) {
  Ws w;
  w.NG = 1;
  w.P = round32(T);
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes); return at; };
  w.status = take(sizeof(int));
  w.counts = take(4 * 2);
  w.cursor = take(4 * 2);
  w.row_start = take(4 * 2);
  w.us_up = take(4 * 2);
  w.us_dn = take(4 * 2);
  w.slot0 = take(4);
  w.xq = take(2 * static_cast<size_t>(w.P) * K_in);
  w.sx = take(4 * static_cast<size_t>(K_in / 128) * w.P);
  if (F > 0) {
    w.hq = take(2 * static_cast<size_t>(w.P) * F);
    w.hs = take(4 * static_cast<size_t>(F / 128) * w.P);
  }
  w.total = o;
  return w;
}

template <class T>
T* at(void* base, size_t off) {
  return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

int check_cfg(const dsmoe_moe_config_t* c) {
  if (!c) return fail(DSMOE_ERR_INVALID, "config is NULL");
  if (c->hidden <= 0 || c->hidden % 128 || c->inter <= 0 || c->inter % 128)
    return fail(DSMOE_ERR_UNSUPPORTED, "hidden (%d) and inter (%d) must be positive multiples of 128", c->hidden,
                c->inter);
  if (c->hidden > 8192 || c->inter > 8192)
    return fail(DSMOE_ERR_UNSUPPORTED, "hidden/inter above 8192 not supported");
  if (c->n_group < 1 || c->n_group > 8 || c->n_routed != 32 * c->n_group)
    return fail(DSMOE_ERR_UNSUPPORTED, "n_routed (%d) must be 32 * n_group with n_group in [1, 8]", c->n_routed);
  if (c->topk_group < 1 || c->topk_group > c->n_group)
    return fail(DSMOE_ERR_INVALID, "topk_group (%d) must be in [1, n_group]", c->topk_group);
  if (c->top_k < 1 || c->top_k > 8 || c->top_k > 32 * c->topk_group)
    return fail(DSMOE_ERR_UNSUPPORTED, "top_k (%d) must be in [1, 8]", c->top_k);
  if (c->router_mode != DSMOE_ROUTER_REF && c->router_mode != DSMOE_ROUTER_V3)
    return fail(DSMOE_ERR_INVALID, "unknown router_mode %d", c->router_mode);
  return DSMOE_OK;
}

int do_route(const dsmoe_moe_config_t* c, const void* hidden, const void* gate, const float* bias, int T,
             int64_t* idx64, float* w_out, const Ws& L, void* ws, cudaStream_t s) {
  if (!hidden || !gate) return fail(DSMOE_ERR_INVALID, "hidden / gate_weight is NULL");
  if (!aligned16(hidden) || !aligned16(gate)) return fail(DSMOE_ERR_INVALID, "hidden / gate_weight not 16-byte aligned");
  if (c->router_mode == DSMOE_ROUTER_V3 && !bias) return fail(DSMOE_ERR_INVALID, "router v3 needs score_bias");
  float* partial = at<float>(ws, L.partial);
  prof(0, s);
  DSMOE_CUDA(launch_router_logits(hidden, gate, partial, T, c->hidden, c->n_routed, L.ksplit, s));
  DSMOE_CUDA(launch_router_select(partial, L.ksplit, bias, T, c->n_routed, c->n_group, c->topk_group, c->top_k,
                                  c->router_mode, c->norm_topk_prob, c->routed_scaling_factor, at<int32_t>(ws, L.idx),
                                  idx64, at<float>(ws, L.w), s));
  if (w_out) DSMOE_CUDA(cudaMemcpyAsync(w_out, at<float>(ws, L.w), sizeof(float) * T * c->top_k,
                                        cudaMemcpyDeviceToDevice, s));
  prof(1, s);
  return DSMOE_OK;
}

int check_weights(const dsmoe_moe_config_t* c, const dsmoe_layer_weights_t* w) {
  if (!w) return fail(DSMOE_ERR_INVALID, "weights is NULL");
  if (w->n_slots < 1) return fail(DSMOE_ERR_INVALID, "n_slots must be >= 1");
  const void* ps[7] = {w->w_gate, w->s_gate, w->w_up, w->s_up, w->w_down, w->s_down, w->slot_of_expert};
  for (const void* p : ps)
    if (!p || !aligned16(p)) return fail(DSMOE_ERR_INVALID, "weight bank pointer NULL or not 16-byte aligned");
  (void)c;
  return DSMOE_OK;
}

// Permute + both grouped GEMMs + combine, routing already in the workspace.
int do_experts(const dsmoe_moe_config_t* c, const dsmoe_layer_weights_t* wt, const void* hidden, int T, void* out,
               const Ws& L, void* ws, cudaStream_t s) {
  const int H = c->hidden, F = c->inter, K = c->top_k, NG = L.NG;
  int32_t* counts = at<int32_t>(ws, L.counts);
  int32_t* row_start = at<int32_t>(ws, L.row_start);
  int32_t* cursor = at<int32_t>(ws, L.cursor);
  int32_t* us_up = at<int32_t>(ws, L.us_up);
  int32_t* us_dn = at<int32_t>(ws, L.us_dn);
  int32_t* idx = at<int32_t>(ws, L.idx);
  uint8_t* xq = at<uint8_t>(ws, L.xq);
  float* sx = at<float>(ws, L.sx);
  uint8_t* hq = at<uint8_t>(ws, L.hq);
  float* hs = at<float>(ws, L.hs);
  __nv_bfloat16* y = at<__nv_bfloat16>(ws, L.y);
  int32_t* pos = at<int32_t>(ws, L.pos);

  DSMOE_CUDA(launch_count(idx, T * K, counts, NG, s));
  DSMOE_CUDA(launch_plan(counts, NG, T, F / 128, H / 128, row_start, cursor, us_up, us_dn, nullptr, s));
  DSMOE_CUDA(launch_quant_scatter(hidden, T, H, idx, K, 1, row_start, cursor, L.P, xq, sx, pos, s));
  prof(2, s);

  CUtensorMap m_w1, m_w3, m_w2, m_x, m_sx, m_h, m_hs;
  int r;
  const uint64_t ns = static_cast<uint64_t>(wt->n_slots);
  if ((r = make_map(&m_w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wt->w_gate, H, ns * F, 128, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_w3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wt->w_up, H, ns * F, 128, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wt->w_down, F, ns * H, 128, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, xq, H, 2ull * L.P, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_sx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, sx, L.P, H / 128, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return r;
  if ((r = make_map(&m_h, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, hq, F, 2ull * L.P, 128, 32, CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_hs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, hs, L.P, F / 128, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return r;

  GemmParams gp{};
  gp.counts = counts;
  gp.row_start = row_start;
  gp.slot_of = wt->slot_of_expert;
  gp.n_groups = NG;
  gp.n_slots = wt->n_slots;
  gp.P = L.P;
  gp.status = at<int>(ws, L.status);
  const int grid = num_sms();

  gp.unit_start = us_up;
  gp.wscale0 = wt->s_gate;
  gp.wscale1 = wt->s_up;
  gp.M = F;
  gp.K = H;
  gp.hq = hq;
  gp.hs = hs;
  DSMOE_CUDA(launch_grouped_gemm(2, m_w1, m_w3, m_x, m_sx, gp, grid, s));
  prof(3, s);

  gp.unit_start = us_dn;
  gp.wscale0 = wt->s_down;
  gp.wscale1 = wt->s_down;
  gp.M = H;
  gp.K = F;
  gp.y = y;
  DSMOE_CUDA(launch_grouped_gemm(1, m_w2, m_w2, m_h, m_hs, gp, grid, s));
  prof(4, s);

  const float scale = c->router_mode == DSMOE_ROUTER_V3 ? 1.0f : c->routed_scaling_factor;
  DSMOE_CUDA(launch_combine(y, T, H, pos, at<float>(ws, L.w), K, row_start, scale,
                            static_cast<__nv_bfloat16*>(out), s));
  prof(5, s);
  return DSMOE_OK;
}

}  // namespace
}  // namespace dsmoe

using namespace dsmoe;

extern "C" {

const char* dsmoe_last_error(void) { return g_err.c_str(); }

int dsmoe_version(void) { return 1; }

int dsmoe_set_profile_events(void* const* events, int32_t n) {
  if (n < 0 || n > kMaxProf || (n > 0 && !events)) return fail(DSMOE_ERR_INVALID, "0 <= n <= %d events", kMaxProf);
  for (int i = 0; i < kMaxProf; ++i) g_prof[i] = i < n ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_nprof = n;
  return DSMOE_OK;
}

size_t dsmoe_workspace_size(const dsmoe_moe_config_t* cfg, int32_t tokens) {
  if (check_cfg(cfg) != DSMOE_OK || tokens < 0) return 0;
  return plan_moe(tokens, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k).total;
}

int dsmoe_route(const dsmoe_moe_config_t* cfg, const void* hidden, const void* gate_weight, const float* score_bias,
                int32_t tokens, int64_t* topk_idx, float* topk_w, void* workspace, size_t workspace_bytes,
                dsmoe_stream_t stream) {
  int r = check_cfg(cfg);
  if (r) return r;
  if (tokens < 0) return fail(DSMOE_ERR_INVALID, "tokens < 0");
  if (tokens == 0) return DSMOE_OK;
  const Ws L = plan_moe(tokens, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k);
  if (!workspace || workspace_bytes < L.total)
    return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, L.total);
  return do_route(cfg, hidden, gate_weight, score_bias, tokens, topk_idx, topk_w, L, workspace,
                  reinterpret_cast<cudaStream_t>(stream));
}

int dsmoe_moe_experts(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden,
                      int32_t tokens, void* out, void* workspace, size_t workspace_bytes, dsmoe_stream_t stream) {
  int r = check_cfg(cfg);
  if (r) return r;
  if ((r = check_weights(cfg, w))) return r;
  if (tokens < 0) return fail(DSMOE_ERR_INVALID, "tokens < 0");
  if (tokens == 0) return DSMOE_OK;
  if (!hidden || !out || !aligned16(hidden) || !aligned16(out))
    return fail(DSMOE_ERR_INVALID, "hidden / out NULL or not 16-byte aligned");
  const Ws L = plan_moe(tokens, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k);
  if (!workspace || workspace_bytes < L.total)
    return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, L.total);
  return do_experts(cfg, w, hidden, tokens, out, L, workspace, reinterpret_cast<cudaStream_t>(stream));
}

int dsmoe_moe_forward(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden,
                      int32_t tokens, void* out, int64_t* topk_idx, float* topk_w, void* workspace,
                      size_t workspace_bytes, dsmoe_stream_t stream) {
  int r = check_cfg(cfg);
  if (r) return r;
  if ((r = check_weights(cfg, w))) return r;
  if (tokens < 0) return fail(DSMOE_ERR_INVALID, "tokens < 0");
  if (tokens == 0) return DSMOE_OK;
  if (!hidden || !out || !aligned16(hidden) || !aligned16(out))
    return fail(DSMOE_ERR_INVALID, "hidden / out NULL or not 16-byte aligned");
  const Ws L = plan_moe(tokens, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k);
  if (!workspace || workspace_bytes < L.total)
    return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, L.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if ((r = do_route(cfg, hidden, w->gate_weight, w->score_bias, tokens, topk_idx, topk_w, L, workspace, s))) return r;
  return do_experts(cfg, w, hidden, tokens, out, L, workspace, s);
}

size_t dsmoe_expert_ffn_workspace_size(int32_t tokens, int32_t hidden, int32_t inter) {
  if (tokens < 0 || hidden <= 0 || inter <= 0) return 0;
  return plan_single(tokens, hidden, inter).total;
}

size_t dsmoe_fp8_linear_workspace_size(int32_t tokens, int32_t in_features, int32_t out_features) {
  if (tokens < 0 || in_features <= 0 || out_features <= 0) return 0;
  return plan_single(tokens, in_features, 0).total;
}

// Shared by dsmoe_expert_ffn and dsmoe_fp8_linear: one group, slot 0.
static int single_prologue(const void* x, int T, int K_in, int mt_up, int mt_dn, const Ws& L, void* ws,
                           cudaStream_t s) {
  DSMOE_CUDA(cudaMemsetAsync(at<int32_t>(ws, L.slot0), 0, 4, s));
  DSMOE_CUDA(launch_plan(at<int32_t>(ws, L.counts), 1, T, mt_up, mt_dn, at<int32_t>(ws, L.row_start),
                         at<int32_t>(ws, L.cursor), at<int32_t>(ws, L.us_up), at<int32_t>(ws, L.us_dn), nullptr, s));
  DSMOE_CUDA(launch_quant_scatter(x, T, K_in, nullptr, 0, 1, at<int32_t>(ws, L.row_start),
                                  at<int32_t>(ws, L.cursor), L.P, at<uint8_t>(ws, L.xq), at<float>(ws, L.sx), nullptr,
                                  s));
  return DSMOE_OK;
}

int dsmoe_expert_ffn(const void* x, int32_t tokens, int32_t hidden, int32_t inter, const void* w_gate,
                     const float* s_gate, const void* w_up, const float* s_up, const void* w_down,
                     const float* s_down, void* out, void* workspace, size_t workspace_bytes,
                     dsmoe_stream_t stream) {
  if (hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || hidden > 8192 || inter > 8192)
    return fail(DSMOE_ERR_UNSUPPORTED, "hidden (%d) / inter (%d) must be multiples of 128 up to 8192", hidden, inter);
  if (tokens < 0) return fail(DSMOE_ERR_INVALID, "tokens < 0");
  if (tokens == 0) return DSMOE_OK;
  const void* ps[9] = {x, w_gate, s_gate, w_up, s_up, w_down, s_down, out, workspace};
  for (const void* p : ps)
    if (!p || !aligned16(p)) return fail(DSMOE_ERR_INVALID, "pointer NULL or not 16-byte aligned");
  const Ws L = plan_single(tokens, hidden, inter);
  if (workspace_bytes < L.total) return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, L.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int r;
  int32_t* counts = at<int32_t>(workspace, L.counts);
  if ((r = single_prologue(x, tokens, hidden, inter / 128, hidden / 128, L, workspace, s))) return r;
  CUtensorMap m_w1, m_w3, m_w2, m_x, m_sx, m_h, m_hs;
  if ((r = make_map(&m_w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w_gate, hidden, inter, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_w3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w_up, hidden, inter, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w_down, inter, hidden, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, at<uint8_t>(workspace, L.xq), hidden, 2ull * L.P, 128, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_sx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, at<float>(workspace, L.sx), L.P, hidden / 128, 128, 1,
                    CU_TENSOR_MAP_SWIZZLE_NONE))) return r;
  if ((r = make_map(&m_h, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, at<uint8_t>(workspace, L.hq), inter, 2ull * L.P, 128, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_hs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, at<float>(workspace, L.hs), L.P, inter / 128, 128, 1,
                    CU_TENSOR_MAP_SWIZZLE_NONE))) return r;
  GemmParams gp{};
  gp.counts = counts;
  gp.row_start = at<int32_t>(workspace, L.row_start);
  gp.slot_of = at<int32_t>(workspace, L.slot0);
  gp.n_groups = 1;
  gp.n_slots = 1;
  gp.P = L.P;
  gp.status = at<int>(workspace, L.status);
  const int grid = num_sms();
  gp.unit_start = at<int32_t>(workspace, L.us_up);
  gp.wscale0 = s_gate;
  gp.wscale1 = s_up;
  gp.M = inter;
  gp.K = hidden;
  gp.hq = at<uint8_t>(workspace, L.hq);
  gp.hs = at<float>(workspace, L.hs);
  DSMOE_CUDA(launch_grouped_gemm(2, m_w1, m_w3, m_x, m_sx, gp, grid, s));
  gp.unit_start = at<int32_t>(workspace, L.us_dn);
  gp.wscale0 = s_down;
  gp.wscale1 = s_down;
  gp.M = hidden;
  gp.K = inter;
  gp.y = static_cast<__nv_bfloat16*>(out);
  DSMOE_CUDA(launch_grouped_gemm(1, m_w2, m_w2, m_h, m_hs, gp, grid, s));
  return DSMOE_OK;
}

int dsmoe_fp8_linear(const void* x, int32_t tokens, int32_t in_features, int32_t out_features, const void* weight,
                     const float* scale_inv, void* out, void* workspace, size_t workspace_bytes,
                     dsmoe_stream_t stream) {
  if (in_features <= 0 || in_features % 128 || out_features <= 0 || out_features % 128 || in_features > 8192)
    return fail(DSMOE_ERR_UNSUPPORTED, "in (%d) / out (%d) features must be multiples of 128 (in <= 8192)",
                in_features, out_features);
  if (tokens < 0) return fail(DSMOE_ERR_INVALID, "tokens < 0");
  if (tokens == 0) return DSMOE_OK;
  const void* ps[5] = {x, weight, scale_inv, out, workspace};
  for (const void* p : ps)
    if (!p || !aligned16(p)) return fail(DSMOE_ERR_INVALID, "pointer NULL or not 16-byte aligned");
  const Ws L = plan_single(tokens, in_features, 0);
  if (workspace_bytes < L.total) return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, L.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int r;
  int32_t* counts = at<int32_t>(workspace, L.counts);
  if ((r = single_prologue(x, tokens, in_features, 0, out_features / 128, L, workspace, s))) return r;
  CUtensorMap m_w, m_x, m_sx;
  if ((r = make_map(&m_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, weight, in_features, out_features, 128, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, at<uint8_t>(workspace, L.xq), in_features, 2ull * L.P,
                    128, 32, CU_TENSOR_MAP_SWIZZLE_128B))) return r;
  if ((r = make_map(&m_sx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, at<float>(workspace, L.sx), L.P, in_features / 128,
                    128, 1, CU_TENSOR_MAP_SWIZZLE_NONE))) return r;
  GemmParams gp{};
  gp.counts = counts;
  gp.row_start = at<int32_t>(workspace, L.row_start);
  gp.slot_of = at<int32_t>(workspace, L.slot0);
  gp.n_groups = 1;
  gp.n_slots = 1;
  gp.P = L.P;
  gp.status = at<int>(workspace, L.status);
  gp.unit_start = at<int32_t>(workspace, L.us_dn);
  gp.wscale0 = scale_inv;
  gp.wscale1 = scale_inv;
  gp.M = out_features;
  gp.K = in_features;
  gp.y = static_cast<__nv_bfloat16*>(out);
  DSMOE_CUDA(launch_grouped_gemm(1, m_w, m_w, m_x, m_sx, gp, num_sms(), s));
  return DSMOE_OK;
}

int dsmoe_read_status(void* workspace, int32_t* device_status, dsmoe_stream_t stream) {
  if (!workspace || !device_status) return fail(DSMOE_ERR_INVALID, "NULL argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  DSMOE_CUDA(cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
  DSMOE_CUDA(cudaStreamSynchronize(s));
  DSMOE_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  *device_status = v;
  return v == 0 ? DSMOE_OK : fail(DSMOE_ERR_DEVICE, "device status %d", v);
}

}  // extern "C"
