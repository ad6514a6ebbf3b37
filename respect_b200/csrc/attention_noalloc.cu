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

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device

// Device-side array; in host code this name is only a handle for
// cudaGetSymbolAddress, never an address a kernel may be given.
static __device__ __align__(256) float g_attn_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
// The array's device address differs per CUDA context (a device's primary
// context, a context the caller created, a context re-created after a device
// reset), so it is looked up with the calling thread's current context and
// cached per context.
using CtxGetCurrent = CUresult (*)(CUcontext*);
std::mutex g_scratch_mu;
CtxGetCurrent g_ctx_get = nullptr;
constexpr int kMaxCtx = 64;
CUcontext g_ctx[kMaxCtx] = {nullptr};
void* g_addr[kMaxCtx] = {nullptr};
int g_nctx = 0;

int current_context(CUcontext* out) {
  if (!g_ctx_get) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return RB_ERR_CUDA;
    g_ctx_get = reinterpret_cast<CtxGetCurrent>(fn);
  }
  *out = nullptr;
  if (g_ctx_get(out) != CUDA_SUCCESS) return RB_ERR_CUDA;
  return RB_OK;
}

// Device address of g_attn_scratch in the current context.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return RB_ERR_CUDA;   // makes the device's primary context current if none is
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  CUcontext ctx = nullptr;
  const int st = current_context(&ctx);
  if (st != RB_OK) return st;
  for (int i = 0; i < g_nctx; ++i)
    if (g_ctx[i] == ctx && ctx != nullptr) {
      *out = g_addr[i];
      return RB_OK;
    }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_attn_scratch) != cudaSuccess || !p) return RB_ERR_CUDA;
  if (ctx != nullptr) {   // remember it (the oldest entry gives way when the table is full)
    const int slot = g_nctx < kMaxCtx ? g_nctx++ : 0;
    g_ctx[slot] = ctx;
    g_addr[slot] = p;
  }
  *out = p;
  return RB_OK;
}
}  // namespace

}  // namespace rb

extern "C" int rb_fused_attn_hyb_noalloc(const rb_attn_args* a, void* stream) {
  using namespace rb;
  const int st = attn_validate(a);
  if (st != RB_OK) return st;
  if (a->M == 0) return RB_OK;
  // Every partial the node phase reads is written earlier in the same call, so
  // the array needs no clearing; it keeps the last call's values.
  if (attn_workspace_bytes(a->H, a->M, a->D, a->NP) > kNoAllocScratchBytes) return RB_ERR_CAPACITY;
  void* ws = nullptr;
  const int r = scratch_address(&ws);
  if (r != RB_OK) return r;
  return attn_launch(a, ws, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}
