// libdsmoe C ABI: argument checks, workspace planning, TMA descriptors and
// the launch sequence of the MoE block. See include/dsmoe.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
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

// Optional cap on the grouped GEMMs' persistent grid (dsmoe_set_gemm_sm_limit),
// per host thread; 0 = one CTA per SM.
thread_local int g_gemm_ctas = 0;

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
// Feature sizes of the single-matrix entry points (dsmoe_expert_ffn,
// dsmoe_fp8_linear): the dense FFN layers need 18432; row offsets stay in int.
constexpr int kMaxFeatures = 32768;
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
  size_t status = 0, counts = 0, cursor = 0, row_start = 0, us_up = 0, us_dn = 0, slot0 = 0, nrows = 0;
  size_t partial = 0, idx = 0, w = 0, pos = 0, xq = 0, sx = 0, gu = 0, hq = 0, hs = 0, y = 0, total = 0;
  int P = 0, ksplit = 1, NG = 1, tile = 32;
};

// Routed MoE block: groups = shared + n_routed; rows = shared segment +
// routed segments, every segment padded to a multiple of 32 rows.
Ws plan_moe(int T, int H, int F, int E, int K) {
  Ws w;
  w.NG = E + 1;
  const long long pairs = static_cast<long long>(T) * K;
  const long long pad = 31LL * (pairs < E ? pairs : E);
  w.P = round32(T) + round32(static_cast<int>(pairs + pad));
  w.ksplit = router_tc_ksplit(T, H, 148);
  w.tile = gemm_tile_tokens(T);
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t at = o; o = align_up(o + bytes); return at; };
  w.status = take(sizeof(int));
  w.counts = take(4 * w.NG);
  w.cursor = take(4 * w.NG);
  w.row_start = take(4 * (w.NG + 1));
  w.us_up = take(4 * (w.NG + 1));
  w.us_dn = take(4 * (w.NG + 1));
  w.slot0 = take(4);
  w.nrows = take(4);
  w.partial = take(sizeof(float) * static_cast<size_t>(w.ksplit) * T * E);
  w.idx = take(4 * static_cast<size_t>(pairs));
  w.w = take(4 * static_cast<size_t>(pairs));
  w.pos = take(4 * static_cast<size_t>(pairs));
  w.xq = take(2 * static_cast<size_t>(w.P) * H);
  w.sx = take(4 * static_cast<size_t>(w.P));
  w.gu = take(2 * static_cast<size_t>(w.P) * 2 * F);
  w.hq = take(2 * static_cast<size_t>(w.P) * F);
  w.hs = take(4 * static_cast<size_t>(w.P));
  w.y = take(2 * static_cast<size_t>(w.P) * H);
  w.total = o;
  return w;
}

// Single expert (or single linear): one group holding every token in order.
Ws plan_single(int T, int K_in, int F /* 0 for a plain linear */) {
  Ws w;
  w.NG = 1;
  w.P = round32(T);
  w.tile = gemm_tile_tokens(T);
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
  w.sx = take(4 * static_cast<size_t>(w.P));
  if (F > 0) {
    w.gu = take(2 * static_cast<size_t>(w.P) * 2 * F);
    w.hq = take(2 * static_cast<size_t>(w.P) * F);
    w.hs = take(4 * static_cast<size_t>(w.P));
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
  CUtensorMap m_x, m_g;
  int r;
  if ((r = make_map(&m_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, hidden, c->hidden, T, 64, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_g, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, gate, c->hidden, c->n_routed, 64, c->n_routed,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  prof(0, s);
  DSMOE_CUDA(launch_router_logits_tc(m_x, m_g, partial, T, c->hidden, c->n_routed, L.ksplit, at<int>(ws, L.status),
                                     s));
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


// One grouped-GEMM launch: TMA descriptors for the weight bank(s), the hi/lo
// activation rows and their scales, then the persistent kernel.
struct GemmJob {
  const void* w0;
  const void* w1;       // second matrix (gate/up), else == w0
  const float* s0;
  const float* s1;
  int n_mat, M, K, n_slots;
  const uint8_t* xq;    // [2P][K] e4m3
  const float* sx;      // [P] per-row scales
  int P;
  const int32_t *counts, *row_start, *unit_start, *slot_of;
  int n_groups;
  int tile;             // token tile (gemm_tile_tokens)
  __nv_bfloat16* y;     // [P][n_mat * M]
  int* status;
};

int run_gemm(const GemmJob& j, cudaStream_t s) {
  CUtensorMap m_w0, m_w1, m_x, m_x32;
  const uint64_t rows = static_cast<uint64_t>(j.n_slots) * j.M;
  int r;
  if ((r = make_map(&m_w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, j.w0, j.K, rows, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, j.w1, j.K, rows, 128, 128, CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_x, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, j.xq, j.K, 2ull * j.P, 128, j.tile,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  if ((r = make_map(&m_x32, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, j.xq, j.K, 2ull * j.P, 128, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B)))
    return r;
  GemmParams gp{};
  gp.counts = j.counts;
  gp.row_start = j.row_start;
  gp.unit_start = j.unit_start;
  gp.slot_of = j.slot_of;
  gp.wscale0 = j.s0;
  gp.wscale1 = j.s1;
  gp.n_groups = j.n_groups;
  gp.n_slots = j.n_slots;
  gp.n_mat = j.n_mat;
  gp.M = j.M;
  gp.K = j.K;
  gp.P = j.P;
  gp.sx = j.sx;
  gp.y = j.y;
  gp.status = j.status;
  const int ctas = g_gemm_ctas > 0 && g_gemm_ctas < num_sms() ? g_gemm_ctas : num_sms();
  DSMOE_CUDA(launch_grouped_gemm(m_w0, m_w1, m_x, m_x32, gp, j.tile, ctas, s));
  return DSMOE_OK;
}

// Gate/up GEMM -> SwiGLU + hi/lo split -> down GEMM, for any group table.
int run_ffn(const void* w_gate, const float* s_gate, const void* w_up, const float* s_up, const void* w_down,
            const float* s_down, int n_slots, int H, int F, const Ws& L, void* ws, const int32_t* slot_of,
            int n_groups, __nv_bfloat16* y, cudaStream_t s) {
  GemmJob j{};
  j.n_slots = n_slots;
  j.P = L.P;
  j.counts = at<int32_t>(ws, L.counts);
  j.row_start = at<int32_t>(ws, L.row_start);
  j.slot_of = slot_of;
  j.n_groups = n_groups;
  j.tile = L.tile;
  j.status = at<int>(ws, L.status);
  int r;
  j.w0 = w_gate;
  j.w1 = w_up;
  j.s0 = s_gate;
  j.s1 = s_up;
  j.n_mat = 2;
  j.M = F;
  j.K = H;
  j.xq = at<uint8_t>(ws, L.xq);
  j.sx = at<float>(ws, L.sx);
  j.unit_start = at<int32_t>(ws, L.us_up);
  j.y = at<__nv_bfloat16>(ws, L.gu);
  if ((r = run_gemm(j, s))) return r;
  prof(3, s);
  DSMOE_CUDA(launch_swiglu_quant(at<__nv_bfloat16>(ws, L.gu), F, at<int32_t>(ws, L.row_start),
                                 at<int32_t>(ws, L.counts), n_groups, L.P, at<uint8_t>(ws, L.hq), at<float>(ws, L.hs),
                                 s));
  prof(4, s);
  j.w0 = j.w1 = w_down;
  j.s0 = j.s1 = s_down;
  j.n_mat = 1;
  j.M = H;
  j.K = F;
  j.xq = at<uint8_t>(ws, L.hq);
  j.sx = at<float>(ws, L.hs);
  j.unit_start = at<int32_t>(ws, L.us_dn);
  j.y = y;
  if ((r = run_gemm(j, s))) return r;
  prof(5, s);
  return DSMOE_OK;
}

// Permute + both grouped GEMMs + combine, routing already in the workspace.
int do_experts(const dsmoe_moe_config_t* c, const dsmoe_layer_weights_t* wt, const void* hidden, int T, void* out,
               const Ws& L, void* ws, cudaStream_t s, const void* residual = nullptr) {
  const int H = c->hidden, F = c->inter, K = c->top_k, NG = L.NG;
  int32_t* counts = at<int32_t>(ws, L.counts);
  int32_t* row_start = at<int32_t>(ws, L.row_start);
  int32_t* cursor = at<int32_t>(ws, L.cursor);
  int32_t* us_up = at<int32_t>(ws, L.us_up);
  int32_t* us_dn = at<int32_t>(ws, L.us_dn);
  int32_t* idx = at<int32_t>(ws, L.idx);
  __nv_bfloat16* y = at<__nv_bfloat16>(ws, L.y);
  int32_t* pos = at<int32_t>(ws, L.pos);

  DSMOE_CUDA(launch_count(idx, T * K, counts, NG, s));
  DSMOE_CUDA(launch_plan(counts, NG, T, L.tile, 2 * F / 128, H / 128, row_start, cursor, us_up, us_dn, s));
  DSMOE_CUDA(launch_quant_scatter(hidden, T, H, idx, K, NG, 1, row_start, cursor, L.P, at<uint8_t>(ws, L.xq),
                                  at<float>(ws, L.sx), pos, s));
  prof(2, s);

  int r;
  if ((r = run_ffn(wt->w_gate, wt->s_gate, wt->w_up, wt->s_up, wt->w_down, wt->s_down, wt->n_slots, H, F, L, ws,
                   wt->slot_of_expert, NG, y, s)))
    return r;

  const float scale = c->router_mode == DSMOE_ROUTER_V3 ? 1.0f : c->routed_scaling_factor;
  DSMOE_CUDA(launch_combine(y, T, H, pos, at<float>(ws, L.w), K, row_start, scale, 1,
                            static_cast<const __nv_bfloat16*>(residual), static_cast<__nv_bfloat16*>(out), s));
  prof(6, s);
  return DSMOE_OK;
}

}  // namespace

int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

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

int dsmoe_clock_probe(uint64_t* out, int32_t n_slots, dsmoe_stream_t stream) {
  if (!out || n_slots < num_sms()) return fail(DSMOE_ERR_INVALID, "clock probe: %d slots for %d SMs", n_slots, num_sms());
  DSMOE_CUDA(launch_clock_probe(reinterpret_cast<unsigned long long*>(out), n_slots, num_sms(),
                                reinterpret_cast<cudaStream_t>(stream)));
  return DSMOE_OK;
}

int dsmoe_set_gemm_sm_limit(int32_t max_ctas) {
  if (max_ctas < 0) return fail(DSMOE_ERR_INVALID, "max_ctas < 0");
  g_gemm_ctas = max_ctas;
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

int dsmoe_rms_norm(const void* x, const void* weight, float eps, int32_t tokens, int32_t hidden, void* out,
                   dsmoe_stream_t stream) {
  if (tokens < 0 || hidden <= 0 || hidden % 8) return fail(DSMOE_ERR_INVALID, "tokens >= 0, hidden > 0 and % 8 == 0");
  if (!(eps >= 0.f)) return fail(DSMOE_ERR_INVALID, "eps must be >= 0");
  if (tokens == 0) return DSMOE_OK;
  if (!x || !weight || !out || !aligned16(x) || !aligned16(weight) || !aligned16(out))
    return fail(DSMOE_ERR_INVALID, "x / weight / out NULL or not 16-byte aligned");
  DSMOE_CUDA(launch_rmsnorm(x, weight, eps, tokens, hidden, out, reinterpret_cast<cudaStream_t>(stream)));
  return DSMOE_OK;
}

int dsmoe_sample_top_p(const float* logits, int32_t rows, int32_t vocab, int64_t row_stride, float temperature,
                       float top_p, const float* uniforms, int64_t* tokens, int32_t* nucleus_sizes,
                       dsmoe_stream_t stream) {
  if (rows < 0 || rows > 65535) return fail(DSMOE_ERR_INVALID, "0 <= rows <= 65535");
  if (vocab < 1 || vocab > top_p_max_vocab())
    return fail(DSMOE_ERR_UNSUPPORTED, "vocab %d outside [1, %d]", vocab, top_p_max_vocab());
  if (row_stride < vocab) return fail(DSMOE_ERR_INVALID, "row_stride < vocab");
  if (!(temperature >= 0.f) || !std::isfinite(temperature))
    return fail(DSMOE_ERR_INVALID, "temperature must be finite and >= 0");
  if (!(top_p >= 0.f)) return fail(DSMOE_ERR_INVALID, "top_p must be >= 0");
  if (rows == 0) return DSMOE_OK;
  if (!logits || !tokens || (temperature > 0.f && !uniforms))
    return fail(DSMOE_ERR_INVALID, "logits / tokens NULL, or uniforms NULL with temperature > 0");
  if (reinterpret_cast<uintptr_t>(logits) % 4 || reinterpret_cast<uintptr_t>(tokens) % 8)
    return fail(DSMOE_ERR_INVALID, "logits / tokens misaligned");
  DSMOE_CUDA(launch_top_p(logits, rows, vocab, row_stride, temperature, top_p, uniforms,
                          reinterpret_cast<long long*>(tokens), nucleus_sizes,
                          reinterpret_cast<cudaStream_t>(stream)));
  return DSMOE_OK;
}

size_t dsmoe_moe_layer_ffn_workspace_size(const dsmoe_moe_config_t* cfg, int32_t tokens) {
  if (check_cfg(cfg) != DSMOE_OK || tokens < 0) return 0;
  const size_t moe = plan_moe(tokens, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k).total;
  return moe + ((static_cast<size_t>(tokens) * cfg->hidden * 2 + 255) & ~size_t(255));
}

int dsmoe_moe_layer_ffn(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden,
                        const void* norm_weight, float eps, int32_t tokens, void* out, int64_t* topk_idx,
                        float* topk_w, void* workspace, size_t workspace_bytes, dsmoe_stream_t stream) {
  int r = check_cfg(cfg);
  if (r) return r;
  if ((r = check_weights(cfg, w))) return r;
  if (tokens < 0) return fail(DSMOE_ERR_INVALID, "tokens < 0");
  if (!(eps >= 0.f)) return fail(DSMOE_ERR_INVALID, "eps must be >= 0");
  if (tokens == 0) return DSMOE_OK;
  if (!hidden || !out || !norm_weight || !aligned16(hidden) || !aligned16(out) || !aligned16(norm_weight))
    return fail(DSMOE_ERR_INVALID, "hidden / norm_weight / out NULL or not 16-byte aligned");
  if (out == hidden) return fail(DSMOE_ERR_INVALID, "out must not alias hidden");
  const Ws L = plan_moe(tokens, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k);
  const size_t need = dsmoe_moe_layer_ffn_workspace_size(cfg, tokens);
  if (!workspace || workspace_bytes < need)
    return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, need);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  void* normed = static_cast<uint8_t*>(workspace) + L.total;  // L.total is a multiple of the 256-byte alignment
  DSMOE_CUDA(launch_rmsnorm(hidden, norm_weight, eps, tokens, cfg->hidden, normed, s));
  if ((r = do_route(cfg, normed, w->gate_weight, w->score_bias, tokens, topk_idx, topk_w, L, workspace, s))) return r;
  return do_experts(cfg, w, normed, tokens, out, L, workspace, s, hidden);
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
  DSMOE_CUDA(launch_plan(at<int32_t>(ws, L.counts), 1, T, L.tile, mt_up, mt_dn, at<int32_t>(ws, L.row_start),
                         at<int32_t>(ws, L.cursor), at<int32_t>(ws, L.us_up), at<int32_t>(ws, L.us_dn), s));
  DSMOE_CUDA(launch_quant_scatter(x, T, K_in, nullptr, 0, 1, 1, at<int32_t>(ws, L.row_start),
                                  at<int32_t>(ws, L.cursor), L.P, at<uint8_t>(ws, L.xq), at<float>(ws, L.sx), nullptr,
                                  s));
  return DSMOE_OK;
}

int dsmoe_expert_ffn(const void* x, int32_t tokens, int32_t hidden, int32_t inter, const void* w_gate,
                     const float* s_gate, const void* w_up, const float* s_up, const void* w_down,
                     const float* s_down, void* out, void* workspace, size_t workspace_bytes,
                     dsmoe_stream_t stream) {
  if (hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || hidden > kMaxFeatures || inter > kMaxFeatures)
    return fail(DSMOE_ERR_UNSUPPORTED, "hidden (%d) / inter (%d) must be multiples of 128 up to %d", hidden, inter,
                kMaxFeatures);
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
  if ((r = single_prologue(x, tokens, hidden, 2 * inter / 128, hidden / 128, L, workspace, s))) return r;
  if ((r = run_ffn(w_gate, s_gate, w_up, s_up, w_down, s_down, 1, hidden, inter, L, workspace,
                   at<int32_t>(workspace, L.slot0), 1, static_cast<__nv_bfloat16*>(out), s)))
    return r;
  return DSMOE_OK;
}

int dsmoe_fp8_linear(const void* x, int32_t tokens, int32_t in_features, int32_t out_features, const void* weight,
                     const float* scale_inv, void* out, void* workspace, size_t workspace_bytes,
                     dsmoe_stream_t stream) {
  if (in_features <= 0 || in_features % 128 || out_features <= 0 || out_features % 8 ||
      in_features > kMaxFeatures || out_features > kMaxFeatures)
    return fail(DSMOE_ERR_UNSUPPORTED,
                "in (%d) features must be a multiple of 128 and out (%d) of 8, both up to %d", in_features,
                out_features, kMaxFeatures);
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
  if ((r = single_prologue(x, tokens, in_features, 0, (out_features + 127) / 128, L, workspace, s))) return r;
  GemmJob j{};
  j.w0 = j.w1 = weight;
  j.s0 = j.s1 = scale_inv;
  j.n_mat = 1;
  j.M = out_features;
  j.K = in_features;
  j.n_slots = 1;
  j.xq = at<uint8_t>(workspace, L.xq);
  j.sx = at<float>(workspace, L.sx);
  j.P = L.P;
  j.counts = counts;
  j.row_start = at<int32_t>(workspace, L.row_start);
  j.unit_start = at<int32_t>(workspace, L.us_dn);
  j.slot_of = at<int32_t>(workspace, L.slot0);
  j.n_groups = 1;
  j.tile = L.tile;
  j.y = static_cast<__nv_bfloat16*>(out);
  j.status = at<int>(workspace, L.status);
  return run_gemm(j, s);
}

// ----------------------------------------------------------- expert parallel
int dsmoe_ep_dispatch(const int64_t* topk_idx, const float* topk_w, const void* hidden, int32_t tokens,
                      int32_t top_k, int32_t hidden_size, int32_t world, int32_t experts_per_rank,
                      int32_t* send_counts, int32_t* tok_rows, int32_t* send_tok, int32_t* send_idx, float* send_w,
                      void* send_hidden, dsmoe_stream_t stream) {
  if (tokens < 0 || top_k < 1 || top_k > 8 || world < 1 || world > 64 || experts_per_rank < 1 || hidden_size <= 0 ||
      hidden_size % 8)
    return fail(DSMOE_ERR_INVALID, "ep_dispatch: bad sizes (tokens %d, top_k %d, world %d, experts/rank %d)", tokens,
                top_k, world, experts_per_rank);
  if (tokens == 0) {
    DSMOE_CUDA(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world, reinterpret_cast<cudaStream_t>(stream)));
    return DSMOE_OK;
  }
  const void* ps[9] = {topk_idx, topk_w, hidden, send_counts, tok_rows, send_tok, send_idx, send_w, send_hidden};
  for (const void* p : ps)
    if (!p) return fail(DSMOE_ERR_INVALID, "ep_dispatch: NULL pointer");
  if (!aligned16(hidden) || !aligned16(send_hidden)) return fail(DSMOE_ERR_INVALID, "ep_dispatch: unaligned rows");
  DSMOE_CUDA(launch_ep_dispatch(topk_idx, topk_w, hidden, tokens, top_k, hidden_size, world, experts_per_rank,
                                send_counts, tok_rows, send_tok, send_idx, send_w, send_hidden,
                                reinterpret_cast<cudaStream_t>(stream)));
  return DSMOE_OK;
}

size_t dsmoe_moe_local_workspace_size(const dsmoe_moe_config_t* cfg, int32_t rows) {
  if (check_cfg(cfg) != DSMOE_OK || rows < 0) return 0;
  return plan_moe(rows, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k).total;
}

// rows_from (optional, peer-memory step): counts_all [world][world] on the
// device; the rows actually received are sum_s counts_all[s][me], counted on
// the device, and `rows` is only the bound that sizes the workspace and grids.
static int moe_local_impl(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden,
                          int32_t rows, const int32_t* local_idx, const float* local_w, void* partial_out,
                          const int32_t* origin, const uint64_t* peer_out, int me, int cap, void* workspace,
                          size_t workspace_bytes, dsmoe_stream_t stream, const int32_t* rows_from = nullptr,
                          int world = 1) {
  int r = check_cfg(cfg);
  if (r) return r;
  if ((r = check_weights(cfg, w))) return r;
  if (rows < 0) return fail(DSMOE_ERR_INVALID, "rows < 0");
  if (rows == 0) return DSMOE_OK;
  if (!hidden || (!partial_out && !peer_out) || !local_idx || !local_w || !aligned16(hidden) ||
      (partial_out && !aligned16(partial_out)) || (peer_out && !origin))
    return fail(DSMOE_ERR_INVALID, "moe_local: NULL or unaligned pointer");
  const Ws L = plan_moe(rows, cfg->hidden, cfg->inter, cfg->n_routed, cfg->top_k);
  if (!workspace || workspace_bytes < L.total)
    return fail(DSMOE_ERR_WORKSPACE, "workspace %zu bytes, need %zu", workspace_bytes, L.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int H = cfg->hidden, F = cfg->inter, K = cfg->top_k, NG = L.NG;
  void* ws = workspace;
  int32_t* counts = at<int32_t>(ws, L.counts);
  int32_t* row_start = at<int32_t>(ws, L.row_start);
  int32_t* pos = at<int32_t>(ws, L.pos);
  int32_t* nrows = nullptr;
  if (rows_from) {
    nrows = at<int32_t>(ws, L.nrows);
    DSMOE_CUDA(launch_ep_recv_rows(rows_from, world, me, nrows, s));
  }
  DSMOE_CUDA(launch_count(local_idx, rows * K, counts, NG, s, nrows, K));
  DSMOE_CUDA(launch_plan(counts, NG, 0, L.tile, 2 * F / 128, H / 128, row_start, at<int32_t>(ws, L.cursor),
                         at<int32_t>(ws, L.us_up), at<int32_t>(ws, L.us_dn), s));
  DSMOE_CUDA(launch_quant_scatter(hidden, rows, H, local_idx, K, NG, 0, row_start, at<int32_t>(ws, L.cursor), L.P,
                                  at<uint8_t>(ws, L.xq), at<float>(ws, L.sx), pos, s, nrows));
  prof(2, s);
  __nv_bfloat16* y = at<__nv_bfloat16>(ws, L.y);
  if ((r = run_ffn(w->w_gate, w->s_gate, w->w_up, w->s_up, w->w_down, w->s_down, w->n_slots, H, F, L, ws,
                   w->slot_of_expert, NG, y, s)))
    return r;
  DSMOE_CUDA(launch_combine(y, rows, H, pos, local_w, K, row_start, 1.0f, 0, nullptr,
                            static_cast<__nv_bfloat16*>(partial_out), s, origin, peer_out, me, cap, nrows));
  prof(6, s);
  return DSMOE_OK;
}

int dsmoe_moe_local(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* hidden, int32_t rows,
                    const int32_t* local_idx, const float* local_w, void* partial_out, void* workspace,
                    size_t workspace_bytes, dsmoe_stream_t stream) {
  return moe_local_impl(cfg, w, hidden, rows, local_idx, local_w, partial_out, nullptr, nullptr, 0, 0, workspace,
                        workspace_bytes, stream);
}

int dsmoe_ep_plan(const int64_t* topk_idx, const float* topk_w, int32_t tokens, int32_t top_k, int32_t world,
                  int32_t experts_per_rank, int32_t* send_counts, int32_t* tok_rows, int32_t* send_tok,
                  int32_t* send_idx, float* send_w, dsmoe_stream_t stream) {
  if (tokens < 0 || top_k < 1 || top_k > 8 || world < 1 || world > 64 || experts_per_rank < 1)
    return fail(DSMOE_ERR_INVALID, "ep_plan: bad sizes (tokens %d, top_k %d, world %d, experts/rank %d)", tokens,
                top_k, world, experts_per_rank);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (tokens == 0) {
    DSMOE_CUDA(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world, s));
    return DSMOE_OK;
  }
  const void* ps[7] = {topk_idx, topk_w, send_counts, tok_rows, send_tok, send_idx, send_w};
  for (const void* p : ps)
    if (!p) return fail(DSMOE_ERR_INVALID, "ep_plan: NULL pointer");
  DSMOE_CUDA(launch_ep_plan(topk_idx, topk_w, tokens, top_k, world, experts_per_rank, send_counts, tok_rows, send_tok,
                            send_idx, send_w, s));
  return DSMOE_OK;
}

int dsmoe_ep_push(const void* hidden, int32_t tokens, int32_t top_k, int32_t hidden_size, int32_t world, int32_t rank,
                  int32_t cap, const int32_t* counts_all, const int32_t* send_tok, const int32_t* send_idx,
                  const float* send_w, int32_t* tok_rows, const uint64_t* peer_recv_hidden,
                  const uint64_t* peer_recv_meta, int32_t* device_status, int32_t max_blocks, dsmoe_stream_t stream) {
  if (tokens < 0 || top_k < 1 || top_k > 8 || world < 1 || world > 64 || rank < 0 || rank >= world ||
      hidden_size <= 0 || hidden_size % 8 || cap < tokens)
    return fail(DSMOE_ERR_INVALID, "ep_push: bad sizes (tokens %d, cap %d, rank %d of %d)", tokens, cap, rank, world);
  if (tokens == 0) return DSMOE_OK;
  const void* ps[8] = {hidden, counts_all, send_tok, send_idx, send_w, tok_rows, peer_recv_hidden, peer_recv_meta};
  for (const void* p : ps)
    if (!p) return fail(DSMOE_ERR_INVALID, "ep_push: NULL pointer");
  if (!aligned16(hidden)) return fail(DSMOE_ERR_INVALID, "ep_push: unaligned rows");
  DSMOE_CUDA(launch_ep_push(hidden, tokens, hidden_size, top_k, world, rank, cap, counts_all, send_tok, send_idx,
                            send_w, tok_rows, peer_recv_hidden, peer_recv_meta, reinterpret_cast<int*>(device_status),
                            max_blocks, reinterpret_cast<cudaStream_t>(stream)));
  return DSMOE_OK;
}

int dsmoe_moe_local_peer(const dsmoe_moe_config_t* cfg, const dsmoe_layer_weights_t* w, const void* recv_hidden,
                         int32_t rows, const int32_t* recv_meta, int32_t world, int32_t rank, int32_t cap,
                         const uint64_t* peer_return, const int32_t* counts_all, void* workspace,
                         size_t workspace_bytes, dsmoe_stream_t stream) {
  if (world < 1 || world > 64 || rank < 0 || rank >= world || cap < 1 || rows < 0 ||
      static_cast<int64_t>(rows) > static_cast<int64_t>(world) * cap)
    return fail(DSMOE_ERR_INVALID, "moe_local_peer: bad sizes (rows %d, cap %d, rank %d of %d)", rows, cap, rank,
                world);
  if (!recv_meta || !peer_return) return fail(DSMOE_ERR_INVALID, "moe_local_peer: NULL pointer");
  const int check = check_cfg(cfg);
  if (check) return check;
  const size_t cap_rows = static_cast<size_t>(world) * cap;
  const int K = cfg->top_k;
  const int32_t* idx = recv_meta;
  const float* wts = reinterpret_cast<const float*>(recv_meta + cap_rows * K);
  const int32_t* origin = recv_meta + 2 * cap_rows * K;
  return moe_local_impl(cfg, w, recv_hidden, rows, idx, wts, nullptr, origin, peer_return, rank, cap, workspace,
                        workspace_bytes, stream, counts_all, world);
}

size_t dsmoe_ep_meta_bytes(int32_t world, int32_t cap, int32_t top_k) {
  if (world < 1 || cap < 1 || top_k < 1) return 0;
  return static_cast<size_t>(world) * cap * (2 * top_k + 2) * sizeof(int32_t);
}

int dsmoe_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  if (!dev_ptr || !handle || bytes == 0) return fail(DSMOE_ERR_INVALID, "ipc_alloc: bad arguments");
  void* p = nullptr;
  DSMOE_CUDA(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(DSMOE_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return DSMOE_OK;
}

int dsmoe_ipc_open(const void* handle, void** dev_ptr) {
  if (!dev_ptr || !handle) return fail(DSMOE_ERR_INVALID, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  DSMOE_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return DSMOE_OK;
}

int dsmoe_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return DSMOE_OK;
  DSMOE_CUDA(cudaIpcCloseMemHandle(dev_ptr));
  return DSMOE_OK;
}

int dsmoe_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return DSMOE_OK;
  DSMOE_CUDA(cudaFree(dev_ptr));
  return DSMOE_OK;
}

int dsmoe_ep_combine(const void* partials, const int32_t* tok_rows, int32_t tokens, int32_t world,
                     int32_t hidden_size, const void* shared_out, float scale, void* out, dsmoe_stream_t stream) {
  if (tokens < 0 || world < 1 || world > 64 || hidden_size <= 0 || hidden_size % 8)
    return fail(DSMOE_ERR_INVALID, "ep_combine: bad sizes");
  if (tokens == 0) return DSMOE_OK;
  if (!tok_rows || !shared_out || !out || !aligned16(shared_out) || !aligned16(out) ||
      (partials && !aligned16(partials)))
    return fail(DSMOE_ERR_INVALID, "ep_combine: NULL or unaligned pointer");
  DSMOE_CUDA(launch_ep_combine(partials, tok_rows, tokens, world, hidden_size, shared_out, scale, out,
                               reinterpret_cast<cudaStream_t>(stream)));
  return DSMOE_OK;
}

int dsmoe_read_status(void* workspace, int32_t* device_status, dsmoe_stream_t stream) {
  if (!device_status) return fail(DSMOE_ERR_INVALID, "NULL argument");
  if (!workspace) {  // the allocation-free entry point's scratch on the current device
    const char* err = "";
    workspace = noalloc_status_word(&err);
    if (!workspace) return fail(DSMOE_ERR_CUDA, "%s", err);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  DSMOE_CUDA(cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
  DSMOE_CUDA(cudaStreamSynchronize(s));
  DSMOE_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  *device_status = v;
  return v == 0 ? DSMOE_OK : fail(DSMOE_ERR_DEVICE, "device status %d", v);
}

}  // extern "C"
