// dsmoe_expert_ffn_noalloc: the single-expert FFN with its scratch memory in a
// fixed device array owned by this library, for callers that cannot allocate
// device memory (see include/dsmoe.h for who they are and the rules).
//
// The array below is a file-scope __device__ variable. Host code must not pass
// its name to a kernel: on the host the name is only a stand-in for the symbol,
// not a device address. The device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and cached.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/dsmoe.h"
#include "kernels.h"

namespace dsmoe {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[DSMOE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of this device's copy of g_noalloc_scratch (set-up on the
// first call per device, with that device current). Returns nullptr and
// fills `err` on failure. `first` tells the caller that this call did the
// set-up.
void* scratch_for_current_device(std::string& err, bool* first = nullptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    err = std::string("cudaGetDevice: ") + cudaGetErrorString(e);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (first) *first = false;
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      err = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e);
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
    if (first) *first = true;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

// The status word is the first int of the scratch (the workspace layout of
// dsmoe_expert_ffn puts it at offset 0).
void* noalloc_status_word(const char** err) {
  static thread_local std::string msg;
  void* p = scratch_for_current_device(msg);
  if (!p && err) *err = msg.c_str();
  return p;
}

}  // namespace dsmoe

extern "C" int dsmoe_expert_ffn_noalloc(const void* x, int32_t tokens, int32_t hidden, int32_t inter,
                                        const void* w_gate, const float* s_gate, const void* w_up,
                                        const float* s_up, const void* w_down, const float* s_down, void* out,
                                        dsmoe_stream_t stream) {
  if (tokens < 0) return dsmoe::set_last_error(DSMOE_ERR_INVALID, "tokens < 0");
  if (tokens == 0) return DSMOE_OK;
  const size_t need = dsmoe_expert_ffn_workspace_size(tokens, hidden, inter);
  if (need > DSMOE_NOALLOC_SCRATCH_BYTES) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "dsmoe_expert_ffn_noalloc: %d tokens x hidden %d x inter %d need %zu bytes of scratch, above the "
             "fixed %d bytes; use dsmoe_expert_ffn with a caller-provided workspace",
             tokens, hidden, inter, need, DSMOE_NOALLOC_SCRATCH_BYTES);
    return dsmoe::set_last_error(DSMOE_ERR_WORKSPACE, buf);
  }
  std::string err;
  bool first = false;
  void* scratch = dsmoe::scratch_for_current_device(err, &first);
  if (!scratch) return dsmoe::set_last_error(DSMOE_ERR_CUDA, err.c_str());
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The device status word at the front is sticky: a kernel records the first
  // error there and only dsmoe_read_status(NULL, ...) reads and clears it, so
  // an error is not lost to the next call. It starts at zero: the set-up
  // clears it once (static device memory is zeroed at load as well). Every
  // other byte whose value can reach `out` is written by a call before it is
  // read; what an earlier call left behind only feeds masked padding columns.
  if (first) {
    const cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(int), s);
    if (e != cudaSuccess) return dsmoe::set_last_error(DSMOE_ERR_CUDA, cudaGetErrorString(e));
  }
  return dsmoe_expert_ffn(x, tokens, hidden, inter, w_gate, s_gate, w_up, s_up, w_down, s_down, out, scratch,
                          DSMOE_NOALLOC_SCRATCH_BYTES, stream);
}
