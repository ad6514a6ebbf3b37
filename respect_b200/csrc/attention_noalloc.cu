// Trie attention for callers that cannot allocate device memory.
//
// rb_fused_attn_hyb needs a scratch buffer for its per-chunk prefix partials,
// which the caller passes in. Some callers have no way to provide one: code
// running where cudaMalloc is off limits (inside a stream capture that must
// not allocate, a host integration whose memory is all pre-planned, a plugin
// that is handed only its input and output buffers). For them this file keeps
// the scratch in a fixed array of device memory that belongs to the library:
// kNoAllocScratchBytes on every GPU that loads the library, held until the
// process exits. The kernels and the results are those of rb_fused_attn_hyb.
#include <mutex>

#include "attention.cuh"
#include "common.cuh"
#include "host_util.h"

namespace rb {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;  // 4 MiB per device

// Device-side array; in host code this name is only a handle for
// cudaGetSymbolAddress, never an address a kernel may be given.
static __device__ __align__(256) float g_attn_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {nullptr};

// Device address of g_attn_scratch on the current device, looked up once per
// device (with that device current) and cached.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return RB_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess || !p) return RB_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return RB_OK;
}
}  // namespace

}  // namespace rb

extern "C" int rb_fused_attn_hyb_noalloc(const rb_attn_args* a, void* stream) {
  using namespace rb;
  const int st = attn_validate(a);
  if (st != RB_OK) return st;
  // Every partial the node phase reads is written earlier in the same call, so
  // the array needs no clearing; it keeps the last call's values.
  if (attn_workspace_bytes(a->H, a->M, a->D, a->NP) > kNoAllocScratchBytes) return RB_ERR_CAPACITY;
  void* ws = nullptr;
  const int r = scratch_address(&ws);
  if (r != RB_OK) return r;
  return attn_launch(a, ws, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}
