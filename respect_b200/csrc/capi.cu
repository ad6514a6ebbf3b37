// extern "C" entry points declared in include/respect_b200.h. Each validates
// its arguments on the host, launches on the caller's stream and returns an
// rb_status; no entry point allocates device memory.
#include "attention.cuh"
#include "common.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "host_util.h"

using namespace rb;

static inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

extern "C" {

const char* rb_status_string(int status) {
  switch (status) {
    case RB_OK: return "ok";
    case RB_ERR_INVALID_ARG: return "invalid argument";
    case RB_ERR_UNSUPPORTED: return "unsupported shape, dtype or layout";
    case RB_ERR_CAPACITY: return "size beyond a fixed capacity";
    case RB_ERR_CUDA: return "CUDA call failed";
    case RB_ERR_DEVICE_TIMEOUT: return "bounded device wait gave up";
    case RB_ERR_WORKSPACE: return "workspace missing or too small";
  }
  return "unknown status";
}

int rb_abi_version(void) { return RB_ABI_VERSION; }

int rb_num_sms(void) { return device_sm_count(); }

int rb_device_error(int* code, int clear) {
  if (!code) return RB_ERR_INVALID_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess) return RB_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return RB_ERR_CUDA;
  *code = v;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)) != cudaSuccess) return RB_ERR_CUDA;
  }
  return RB_OK;
}

// ------------------------------------------------------------------ attention
size_t rb_fused_attn_hyb_workspace(int H, int M, int D, int NP) {
  return attn_workspace_bytes(H, M, D, NP);
}

int rb_fused_attn_hyb(const rb_attn_args* a, void* workspace, size_t ws_bytes, void* stream) {
  return attn_launch(a, workspace, ws_bytes, as_stream(stream));
}

// ------------------------------------------------------------------ linear
size_t rb_linear_workspace(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const GemmShape s = gemm_plan(M, N, K, device_sm_count());
  return s.splits > 1 ? static_cast<size_t>(s.splits) * M * N * sizeof(float) : 0;
}

int rb_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo,
              int out_dtype, int M, int N, int K, void* workspace, size_t ws_bytes, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || !x || !w || !out) return RB_ERR_INVALID_ARG;
  if (out_dtype != RB_BF16 && out_dtype != RB_F32) return RB_ERR_UNSUPPORTED;
  if (M == 0) return RB_OK;
  if (K % 8 != 0 || ldx % 8 != 0 || ldw % 8 != 0 || ldx < K || ldw < K || ldo < N) return RB_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return RB_ERR_UNSUPPORTED;
  const GemmShape s = gemm_plan(M, N, K, device_sm_count());
  GemmLaunch a{};
  a.x = x; a.ldx = ldx; a.w = w; a.ldw = ldw; a.out = out; a.ldo = ldo;
  cudaStream_t st = as_stream(stream);
  if (s.splits == 1) {
    a.epi = out_dtype == RB_F32 ? kEpiStoreF32 : kEpiStoreBF16;
    return gemm_launch(s, a, st);
  }
  const size_t need = static_cast<size_t>(s.splits) * M * N * sizeof(float);
  if (!workspace || ws_bytes < need || !aligned16(workspace)) return RB_ERR_WORKSPACE;
  a.epi = kEpiPartial;
  a.partial = static_cast<float*>(workspace);
  int r = gemm_launch(s, a, st);
  if (r != RB_OK) return r;
  return splitk_reduce(a.partial, s.splits, M, N, out, ldo, out_dtype == RB_F32, st);
}

int rb_linear_swiglu_packed(const void* x, int64_t ldx, const void* w_gu, void* out, int64_t ldo, int M, int F,
                            int K, void* stream) {
  if (M < 0 || F <= 0 || K <= 0 || !x || !w_gu || !out) return RB_ERR_INVALID_ARG;
  if (M == 0) return RB_OK;
  if (F % 128 != 0 || K % 8 != 0 || ldx % 8 != 0 || ldx < K || ldo < F || ldo % 8 != 0) return RB_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(w_gu) || !aligned16(out)) return RB_ERR_UNSUPPORTED;
  const GemmShape s = gemm_plan(M, 2 * F, K, device_sm_count(), 256, 1);
  CUtensorMap mx, mw;
  int r = gemm_encode_x(&mx, x, M, K, ldx);
  if (r != RB_OK) return r;
  r = gemm_encode_w_packed(&mw, w_gu, 2 * F, K, 256);
  if (r != RB_OK) return r;
  GemmLaunch a{};
  a.x = x; a.ldx = ldx; a.w = w_gu; a.out = out; a.ldo = ldo; a.w_tiled = 1;
  a.epi = kEpiSiluMul;
  return gemm_launch_maps(s, mx, mw, a, as_stream(stream));
}

int rb_linear_bn(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  return gemm_plan(1, N, K, device_sm_count()).BN;
}

size_t rb_linear_packed_bytes(int N, int K, int BN) {
  if (N <= 0 || K <= 0) return 0;
  if (BN <= 0) BN = rb_linear_bn(N, K);
  return gemm_packed_elems(N, K, BN) * 2;
}

int rb_pack_linear_weight(const void* w, int64_t ldw, int N, int K, int BN, void* out, void* stream) {
  if (BN <= 0) BN = rb_linear_bn(N, K);
  return gemm_pack_weight(w, ldw, N, K, BN, out, as_stream(stream));
}

int rb_linear_packed(const void* x, int64_t ldx, const void* wp, void* out, int64_t ldo, int out_dtype, int M, int N,
                     int K, void* workspace, size_t ws_bytes, void* stream) {
  if (M < 0 || N <= 0 || K <= 0 || !x || !wp || !out) return RB_ERR_INVALID_ARG;
  if (out_dtype != RB_BF16 && out_dtype != RB_F32) return RB_ERR_UNSUPPORTED;
  if (M == 0) return RB_OK;
  if (K % 8 != 0 || ldx % 8 != 0 || ldx < K || ldo < N) return RB_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(wp) || !aligned16(out)) return RB_ERR_UNSUPPORTED;
  const GemmShape s = gemm_plan(M, N, K, device_sm_count());
  CUtensorMap mx, mw;
  int r = gemm_encode_x(&mx, x, M, K, ldx);
  if (r != RB_OK) return r;
  r = gemm_encode_w_packed(&mw, wp, N, K, s.BN);
  if (r != RB_OK) return r;
  GemmLaunch a{};
  a.x = x; a.ldx = ldx; a.w = wp; a.out = out; a.ldo = ldo; a.w_tiled = 1;
  cudaStream_t st = as_stream(stream);
  if (s.splits == 1) {
    a.epi = out_dtype == RB_F32 ? kEpiStoreF32 : kEpiStoreBF16;
    return gemm_launch_maps(s, mx, mw, a, st);
  }
  const size_t need = static_cast<size_t>(s.splits) * M * N * sizeof(float);
  if (!workspace || ws_bytes < need || !aligned16(workspace)) return RB_ERR_WORKSPACE;
  a.epi = kEpiPartial;
  a.partial = static_cast<float*>(workspace);
  r = gemm_launch_maps(s, mx, mw, a, st);
  if (r != RB_OK) return r;
  return splitk_reduce(a.partial, s.splits, M, N, out, ldo, out_dtype == RB_F32, st);
}

// ------------------------------------------------------------------ rmsnorm / rope / silu
int rb_rmsnorm(const void* x, const void* w, void* y, int M, int N, float eps, int x_dtype, int w_dtype,
               void* stream) {
  if (M < 0 || N <= 0 || !x || !w || !y) return RB_ERR_INVALID_ARG;
  return rmsnorm_launch(x, w, y, M, N, eps, x_dtype, w_dtype, as_stream(stream));
}

int rb_rope(const void* x, int64_t sxb, int64_t sxh, int64_t sxl, int64_t sxd, const void* cos,
            const void* sin, int64_t scb, int64_t scl, void* y, int B, int H, int L, int D, int x_dtype,
            int cs_dtype, int y_dtype, void* stream) {
  if (B < 0 || H < 0 || L < 0 || D <= 0 || (D & 1) || !x || !cos || !sin || !y) return RB_ERR_INVALID_ARG;
  return rope_launch(x, sxb, sxh, sxl, sxd, cos, sin, scb, scl, y, B, H, L, D, x_dtype, cs_dtype, y_dtype,
                     as_stream(stream));
}

int rb_add_sq(const void* r, const void* h, void* x, float* sq, int64_t n, int r_dtype, int h_dtype, int x_dtype,
              void* stream) {
  if (n < 0 || !r || !sq || (h && !x)) return RB_ERR_INVALID_ARG;
  for (int t : {r_dtype, h ? h_dtype : RB_F32, h ? x_dtype : RB_F32})
    if (t != RB_F32 && t != RB_BF16) return RB_ERR_UNSUPPORTED;
  return add_sq_launch(r, h, x, sq, n, r_dtype, h_dtype, x_dtype, as_stream(stream));
}

int rb_norm_apply(const void* x, const float* var, const void* w, void* y, int64_t M, int N, float eps, int x_dtype,
                  int w_dtype, int y_dtype, void* stream) {
  if (M < 0 || N <= 0 || !x || !var || !w || !y) return RB_ERR_INVALID_ARG;
  for (int t : {x_dtype, w_dtype, y_dtype})
    if (t != RB_F32 && t != RB_BF16) return RB_ERR_UNSUPPORTED;
  return norm_apply_launch(x, var, w, y, M, N, eps, x_dtype, w_dtype, y_dtype, as_stream(stream));
}

int rb_silu_mul(const void* g, const void* u, void* y, int64_t n, int dtype, void* stream) {
  if (n < 0 || (n > 0 && (!g || !u || !y))) return RB_ERR_INVALID_ARG;
  return silu_mul_launch(g, u, y, n, dtype, as_stream(stream));
}

// ------------------------------------------------------------------ decode helpers
int rb_greedy_token(const void* logits, int dtype, int64_t ld, int M, int V, int offset, int size,
                    int64_t* out, void* stream) {
  if (M < 0 || V <= 0 || ld < V || !logits || !out || size < 0) return RB_ERR_INVALID_ARG;
  return greedy_launch(logits, dtype, ld, M, V, offset, size, out, as_stream(stream));
}

int rb_compact_kv(void* const* k_layers, void* const* v_layers, int n_layers, int HK, int D, int64_t s_head,
                  int64_t s_slot, int elem_bytes, const int32_t* src_slots, int n, int dst_start, void* stream) {
  if (!k_layers || !v_layers || (n > 0 && !src_slots) || HK <= 0 || D <= 0 || n < 0 || dst_start < 0)
    return RB_ERR_INVALID_ARG;
  if (elem_bytes != 2 && elem_bytes != 4) return RB_ERR_UNSUPPORTED;
  return compact_launch(k_layers, v_layers, n_layers, HK, D, s_head, s_slot, elem_bytes, src_slots, n, dst_start,
                        as_stream(stream));
}

int rb_trie_node_mask(const int32_t* parents, int q, int committed, int M, int NN, uint8_t* msk, int64_t ld,
                      void* stream) {
  if (q < 0 || committed < 0 || M < q || NN < committed + q || ld < NN || !msk || (q > 0 && !parents))
    return RB_ERR_INVALID_ARG;
  return trie_node_mask_launch(parents, q, committed, M, NN, msk, ld, as_stream(stream));
}

int rb_verify_mask(const int32_t* parents, int q, int start, int width, void* mask_bf16, void* stream) {
  if (q < 0 || start < 0 || width < start + q || !mask_bf16 || (q > 0 && !parents)) return RB_ERR_INVALID_ARG;
  return verify_mask_launch(parents, q, start, width, mask_bf16, as_stream(stream));
}

}  // extern "C"
