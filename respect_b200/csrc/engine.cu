// Native verify-step engine: one forward of a Qwen3-style decoder over the
// nodes of a trie, with the dedicated kernels, as respect/decoding/verify.py:12-46
// runs it through HF with respect/kernels/patch.py:70-107 installed.
//
// Per layer (HF Qwen3VLTextDecoderLayer order, PyTorch rounding points):
//   xn = rmsnorm(h)                       (fused into the previous finish kernel)
//   qkv = xn @ Wqkv^T                     split-K tcgen05 GEMM -> fp32 partials
//   q,k = rope(rmsnorm_head(bf16 qkv))    qkv_finish: fixed-order split sum, per-head
//   v   = bf16 qkv                        norm, RoPE, K/V written to their slots
//   a   = trie attention                  prefix chunks + committed + ancestors
//   h   = bf16(h + bf16(a @ Wo^T))        o GEMM + resid_finish (+ post-attn norm)
//   act = silu(bf16 g) * bf16 u           gate/up GEMM with the SiLU*mul epilogue
//   h   = bf16(h + bf16(act @ Wd^T))      down GEMM + resid_finish (+ next norm)
// then logits = final_norm(h) @ Wlm^T in fp32 and the greedy choice per row.
//
// Every reduction has an order fixed by the shapes alone, and each fused
// kernel uses the reduction structure of the standalone operator it replaces,
// so an engine step is bitwise equal to composing rb_linear / rb_rmsnorm /
// rb_rope / rb_silu_mul / rb_fused_attn_hyb, and a row's results never depend
// on how many rows the step carries.
#include <climits>
#include <map>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "host_util.h"

namespace rb {

// ------------------------------------------------------------------ kernels
// Row RMSNorm pieces shared with rmsnorm_kernel (elementwise.cu): thread t of
// NT owns elements t, t+NT, ...; fmaf chain in that order, warp tree, lane-0
// broadcast, warps summed in ascending order.
template <int NT>
__device__ __forceinline__ float row_inv_rms(const float* v, int cnt, int N, float eps, float* red) {
  float ss = 0.f;
  for (int k = 0; k < cnt; ++k) ss = fmaf(v[k], v[k], ss);
  ss = warp_sum(ss);
  ss = __shfl_sync(0xffffffffu, ss, 0);
  const int t = threadIdx.x;
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) tot += red[i];
  return rsqrtf(tot / static_cast<float>(N) + eps);
}

constexpr int kMaxPerThread = 32;  // hidden <= 32 * NT (NT = 1024 for hidden >= 2048)
constexpr int kMaxChainRows = 1024;  // max_rows limit of an engine


// h[row] = embed[ids[row]];  xn[row] = rmsnorm(h[row], w). EPT: elements per thread.
// Also the row's ancestor chain for the attention node phase of every layer:
// chain[row * ld + t] = the ancestor at depth t (t = 0 root .. depth[row] = row),
// walked once per step from the parent array (parents precede children).
template <int NT, int EPT>
__global__ void __launch_bounds__(NT) embed_norm_kernel(const StepParams* __restrict__ sp, const int32_t* __restrict__ ids,
                                                        const uint16_t* __restrict__ emb, const uint16_t* __restrict__ w,
                                                        uint16_t* __restrict__ h, uint16_t* __restrict__ xn, int N,
                                                        int vocab, float eps, const int32_t* __restrict__ parents,
                                                        const int32_t* __restrict__ depths, int32_t* __restrict__ chain,
                                                        int chain_ld) {
  __shared__ float red[NT / 32];
  __shared__ int par_s[kMaxChainRows];
  const int row = blockIdx.x;
  pdl_trigger();
  pdl_wait();
  if (row >= sp->q) return;
  for (int i = threadIdx.x; i <= row && i < kMaxChainRows; i += NT) par_s[i] = parents[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    int dd = depths[row];
    if (dd < 0 || dd > row || dd >= chain_ld || row >= kMaxChainRows) {
      raise_device_error(0x201);
      dd = -1;
    }
    int a = row;
    for (int t = dd; t >= 0; --t) {
      chain[static_cast<int64_t>(row) * chain_ld + t] = a;
      const int par = par_s[a];
      if ((t > 0 && (par < 0 || par >= a)) || (t == 0 && par != -1)) {
        raise_device_error(0x202);  // parents / depths inconsistent
        break;
      }
      a = par;
    }
  }
  int id = ids[row];
  if (id < 0 || id >= vocab) {
    raise_device_error(0x301);
    id = 0;
  }
  const uint16_t* er = emb + static_cast<int64_t>(id) * N;
  // element k of this thread: NT = 1024 rows use the vector ownership of
  // rmsnorm_kernel (4-column groups), narrower rows the strided one
  auto elem = [](int k) { return NT == 1024 ? 4 * (threadIdx.x + (k >> 2) * NT) + (k & 3) : threadIdx.x + k * NT; };
  float v[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int i = elem(k);
    v[k] = 0.f;
    if (i < N) {
      const uint16_t b = er[i];
      h[static_cast<int64_t>(row) * N + i] = b;
      v[k] = bf16_bits_to_f32(b);
    }
  }
  const float r = row_inv_rms<NT>(v, EPT, N, eps, red);
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int i = elem(k);
    if (i < N) {
      const float xh = round_bf16(v[k] * r);
      xn[static_cast<int64_t>(row) * N + i] = f32_to_bf16_bits(bf16_bits_to_f32(w[i]) * xh);
    }
  }
}

// o = bf16(sum_s partial[s]);  h = bf16(h + o);  xn = rmsnorm(h, w)
// Splits are summed in ascending order (as splitk_reduce does). Beyond 8
// splits the split loads of two columns are in flight together, not all of
// them: with the 40-register cap that keeps the block from spilling, and the
// cap lets the CTA of the next (weight-streaming) GEMM fit on the SM beside it
// and start its weight stream while this kernel runs (with every load in
// flight the block took the whole register file).
template <int NT, int EPT, int MAXS>
__global__ void __maxnreg__(40) resid_norm_kernel(const StepParams* __restrict__ sp, const float* __restrict__ part,
                                                        int splits, int M, uint16_t* __restrict__ h,
                                                        const uint16_t* __restrict__ w, uint16_t* __restrict__ xn, int N,
                                                        float eps) {
  __shared__ float red[NT / 32];
  const int row = blockIdx.x;
  pdl_trigger();
  uint16_t wv[EPT];  // the norm weights never change: read before waiting for the GEMM
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int i = threadIdx.x + k * NT;
    wv[k] = i < N ? w[i] : 0;
  }
  pdl_wait();
  if (row >= sp->q) return;
  const int64_t plane = static_cast<int64_t>(M) * N;
  const float* p = part + static_cast<int64_t>(row) * N + threadIdx.x;
  float acc[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    // all splits' loads first (independent), then the sum in ascending split order
    float t[MAXS];
    const bool live = threadIdx.x + k * NT < N;
#pragma unroll
    for (int s = 0; s < MAXS; ++s) t[s] = (live && s < splits) ? p[s * plane + k * NT] : 0.f;
    float a = t[0];
#pragma unroll
    for (int s = 1; s < MAXS; ++s)
      if (s < splits) a += t[s];
    acc[k] = a;
    if (MAXS > 8 && (k & 1)) asm volatile("" ::: "memory");  // no later column's loads hoisted above this point
  }
  float v[EPT];
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int i = threadIdx.x + k * NT;
    v[k] = 0.f;
    if (i < N) {
      const int64_t idx = static_cast<int64_t>(row) * N + i;
      const float hn = round_bf16(bf16_bits_to_f32(h[idx]) + round_bf16(acc[k]));
      h[idx] = f32_to_bf16_bits(hn);
      v[k] = hn;
    }
  }
  const float r = row_inv_rms<NT>(v, EPT, N, eps, red);
#pragma unroll
  for (int k = 0; k < EPT; ++k) {
    const int i = threadIdx.x + k * NT;
    if (i < N) {
      const float xh = round_bf16(v[k] * r);
      xn[static_cast<int64_t>(row) * N + i] = f32_to_bf16_bits(bf16_bits_to_f32(wv[k]) * xh);
    }
  }
}

// resid_norm_kernel for NT = 1024 rows in the vector ownership of
// rmsnorm_kernel: thread t owns the 4-column groups 4(t + j NT) .. +3
// (j < G4). A group's split partials are read as float4, kSplitBatch splits
// in flight at once (one round of loads for up to kSplitBatch splits) and
// added in ascending split order, as in the scalar kernel; h and xn move as
// 8-byte groups. Same 40-register cap, for the same co-residency reason.
constexpr int kSplitBatch = 5;
template <int G4>
__global__ void __maxnreg__(40) resid_norm_vec_kernel(const StepParams* __restrict__ sp, const float* __restrict__ part,
                                                      int splits, int M, uint16_t* __restrict__ h,
                                                      const uint16_t* __restrict__ w, uint16_t* __restrict__ xn, int N,
                                                      float eps) {
  constexpr int NT = 1024;
  __shared__ float red[NT / 32];
  const int row = blockIdx.x;
  pdl_trigger();
  uint16_t wv[4 * G4];  // the norm weights never change: read before waiting for the GEMM
#pragma unroll
  for (int j = 0; j < G4; ++j) {
    const int i = 4 * (threadIdx.x + j * NT);
#pragma unroll
    for (int c = 0; c < 4; ++c) wv[4 * j + c] = i < N ? w[i + c] : 0;
  }
  pdl_wait();
  if (row >= sp->q) return;
  const int64_t plane = static_cast<int64_t>(M) * N;
  float v[4 * G4];
#pragma unroll
  for (int j = 0; j < G4; ++j) {
    const int i = 4 * (threadIdx.x + j * NT);
    const bool live = i < N;
    const float4* p = reinterpret_cast<const float4*>(part + static_cast<int64_t>(row) * N + i);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < splits; s0 += kSplitBatch) {
      float4 t[kSplitBatch];
#pragma unroll
      for (int b = 0; b < kSplitBatch; ++b)
        t[b] = (live && s0 + b < splits) ? __ldcg(p + (s0 + b) * (plane / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int b = 0; b < kSplitBatch; ++b) {
        if (s0 + b >= splits) break;
        if (s0 + b == 0) {
          acc = t[0];
        } else {
          acc.x += t[b].x; acc.y += t[b].y; acc.z += t[b].z; acc.w += t[b].w;
        }
      }
    }
    v[4 * j] = v[4 * j + 1] = v[4 * j + 2] = v[4 * j + 3] = 0.f;
    if (live) {
      uint2* hp = reinterpret_cast<uint2*>(h + static_cast<int64_t>(row) * N + i);
      const uint2 hb = *hp;
      const float a[4] = {acc.x, acc.y, acc.z, acc.w};
      const uint32_t hw[4] = {hb.x & 0xffffu, hb.x >> 16, hb.y & 0xffffu, hb.y >> 16};
#pragma unroll
      for (int c = 0; c < 4; ++c)
        v[4 * j + c] = round_bf16(bf16_bits_to_f32(static_cast<uint16_t>(hw[c])) + round_bf16(a[c]));
      *hp = make_uint2(pack_bf16x2(v[4 * j], v[4 * j + 1]), pack_bf16x2(v[4 * j + 2], v[4 * j + 3]));
    }
  }
  const float r = row_inv_rms<NT>(v, 4 * G4, N, eps, red);
#pragma unroll
  for (int j = 0; j < G4; ++j) {
    const int i = 4 * (threadIdx.x + j * NT);
    if (i < N) {
      float y[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) y[c] = bf16_bits_to_f32(wv[4 * j + c]) * round_bf16(v[4 * j + c] * r);
      *reinterpret_cast<uint2*>(xn + static_cast<int64_t>(row) * N + i) =
          make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
    }
  }
}

// One warp per (row, head) of the fused q|k|v projection output (D = 128,
// lane owns d = lane + 32k). q/k heads: per-head RMSNorm with the reduction of
// rmsnorm_kernel<NT=32>, then RoPE at the node's rotary position; v: copy.
__global__ void __launch_bounds__(128) qkv_finish_kernel(
    const StepParams* __restrict__ sp, const int32_t* __restrict__ depths, const float* __restrict__ part,
    int splits, int M, int H, int HK, const uint16_t* __restrict__ qn_w, const uint16_t* __restrict__ kn_w,
    const uint16_t* __restrict__ cos_t, const uint16_t* __restrict__ sin_t, int max_pos, float eps,
    uint16_t* __restrict__ qbuf, uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, int64_t kv_s_head,
    int max_slots) {
  constexpr int D = 128;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x;
  const int head = blockIdx.y * 4 + warp;
  const int nh = H + 2 * HK;
  pdl_trigger();
  if (row >= sp->q || head >= nh) return;
  // Before the wait: the norm weights and the rotary rows (StepParams and the
  // depths are copied in before the step's first kernel).
  const int slot = sp->prompt_len + sp->base + row;
  const bool vhead = head >= H + HK;
  float wq[4] = {0.f, 0.f, 0.f, 0.f}, cr[4] = {0.f, 0.f, 0.f, 0.f}, sr[4] = {0.f, 0.f, 0.f, 0.f};
  if (!vhead) {
    const uint16_t* w = head < H ? qn_w : kn_w;
    int pos = sp->prompt_len + sp->base + depths[row] + sp->rope_delta;
    if (pos < 0 || pos >= max_pos) {
      raise_device_error(0x303);
      pos = 0;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int d = lane + 32 * k;
      wq[k] = bf16_bits_to_f32(w[d]);
      cr[k] = bf16_bits_to_f32(cos_t[static_cast<int64_t>(pos) * D + d]);
      sr[k] = bf16_bits_to_f32(sin_t[static_cast<int64_t>(pos) * D + d]);
    }
  }
  pdl_wait();
  if (slot >= max_slots) {
    raise_device_error(0x302);
    return;
  }
  const int N = nh * D;
  const int64_t plane = static_cast<int64_t>(M) * N;
  float x[4];
  const float* p = part + static_cast<int64_t>(row) * N + head * D + lane;
#pragma unroll
  for (int k = 0; k < 4; ++k) x[k] = p[32 * k];
  for (int s = 1; s < splits; ++s) {
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] += p[s * plane + 32 * k];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) x[k] = round_bf16(x[k]);
  if (vhead) {  // v head
    uint16_t* dst = vc + (head - H - HK) * kv_s_head + static_cast<int64_t>(slot) * D;
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = f32_to_bf16_bits(x[k]);
    return;
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) ss = fmaf(x[k], x[k], ss);
  ss = warp_sum(ss);
  ss = __shfl_sync(0xffffffffu, ss, 0);
  const float r = rsqrtf((0.f + ss) / static_cast<float>(D) + eps);
  float y[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) y[k] = round_bf16(wq[k] * round_bf16(x[k] * r));
  float o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float xr = k < 2 ? -y[k + 2] : y[k - 2];  // rotate_half: d < 64 takes -x[d+64]
    const float a = round_bf16(__fmul_rn(y[k], cr[k]));
    const float b = round_bf16(__fmul_rn(xr, sr[k]));
    o[k] = round_bf16(__fadd_rn(a, b));
  }
  uint16_t* dst;
  if (head < H) dst = qbuf + (static_cast<int64_t>(head) * M + row) * D;
  else dst = kc + (head - H) * kv_s_head + static_cast<int64_t>(slot) * D;
#pragma unroll
  for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = f32_to_bf16_bits(o[k]);
}

// Greedy ids of the live rows from the per-row keys the lm_head epilogue (or
// the small-vocabulary path below) folded with atomicMax.
// Keys are reset to zero here, ready for the next step (zeroed once at set-up).
__global__ void greedy_finalize_kernel(const StepParams* __restrict__ sp, unsigned long long* __restrict__ keys,
                                       int64_t* __restrict__ out, int rows) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  pdl_trigger();
  pdl_wait();
  if (row >= rows) return;
  const unsigned long long k = keys[row];
  keys[row] = 0;
  if (row >= sp->q) return;
  out[row] = k ? static_cast<int64_t>(0xFFFFFFFFu - static_cast<unsigned int>(k & 0xFFFFFFFFu)) : 0;
}

// Small vocabularies (lm_head split over K): the same keys from the reduced logits.
__global__ void argmax_keys_kernel(const StepParams* __restrict__ sp, const float* __restrict__ logits, int64_t ld,
                                   int V, unsigned long long* __restrict__ keys) {
  const int row = blockIdx.y;
  pdl_trigger();
  pdl_wait();
  if (row >= sp->q) return;
  const int ex0 = sp->act_off, ex1 = sp->act_off + sp->act_size;
  unsigned long long best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x)
    if (i < ex0 || i >= ex1) {
      const unsigned long long k = argmax_key(logits[static_cast<int64_t>(row) * ld + i], i);
      best = k > best ? k : best;
    }
  if (best) atomicMax(keys + row, best);
}

}  // namespace rb

// ------------------------------------------------------------------ host engine
using namespace rb;

// ------------------------------------------------------------ acceptance on the device
// The acceptance walk of respect/decoding/acceptance.py:26-46 over the step's
// trie and greedy picks, without the host: node j is accepted iff its root
// holds `first`, every node below the root holds the pick after its parent,
// no strict ancestor holds `eos`, and depth(j) < cap (parents precede
// children, a node has at most one child per token, so the accepted nodes form
// one chain, one per depth). Record: [count, correction, base, prompt_len,
// path[max_rows], tokens[max_rows]]; the correction is the pick after the last
// accepted node (eos when that node is eos; `first` when nothing is accepted).
constexpr int kAcceptHdr = 4;
__global__ void __launch_bounds__(1024) accept_kernel(const StepParams* __restrict__ sp, const int32_t* __restrict__ ids,
                                                      const int32_t* __restrict__ parents,
                                                      const int32_t* __restrict__ depths,
                                                      const int64_t* __restrict__ picks, int first, int cap, int eos,
                                                      int max_rows, int32_t* __restrict__ rec) {
  __shared__ int32_t s_ids[kMaxChainRows], s_par[kMaxChainRows], s_pick[kMaxChainRows], s_path[kMaxChainRows];
  const int q = min(sp->q, kMaxChainRows);
  for (int j = threadIdx.x; j < q; j += blockDim.x) {
    s_ids[j] = ids[j];
    s_par[j] = parents[j];
    s_pick[j] = static_cast<int32_t>(picks[j]);
    s_path[j] = INT_MAX;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < q; j += blockDim.x) {
    const int d = depths[j];
    if (d < 0 || d >= cap || d >= q) continue;
    bool ok = true;
    int c = j, steps = 0;
    while (ok) {
      const int par = s_par[c];
      if (par < 0) {
        ok = s_ids[c] == first && steps == d;
        break;
      }
      if (par >= c || steps >= d) {  // malformed trie (the host validates it): accept nothing here
        ok = false;
        break;
      }
      ok = s_ids[c] == s_pick[par] && s_ids[par] != eos;
      c = par;
      ++steps;
    }
    if (ok) atomicMin(&s_path[d], j);  // one node per depth in a valid trie; lowest index otherwise
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int lim = min(cap, q);
    int n = 0;
    while (n < lim && s_path[n] != INT_MAX) ++n;
    int corr = first;
    if (n > 0) {
      const int last = s_path[n - 1];
      corr = s_ids[last] == eos ? eos : s_pick[last];
    }
    rec[0] = n;
    rec[1] = corr;
    rec[2] = sp->base;
    rec[3] = sp->prompt_len;
  }
  __syncthreads();
  const int n = rec[0];
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    rec[kAcceptHdr + i] = s_path[i];
    rec[kAcceptHdr + max_rows + i] = s_ids[s_path[i]];
  }
}

// kv_buffer.py:93-104 driven by the acceptance record: slot PL + base + path[i]
// moves to PL + base + i for every layer, head, K and V (each thread moves one
// 16-byte piece of every accepted slot, in ascending order, so the moves that
// overlap read their source before it is overwritten).
struct KvLayers {
  void* k[RB_COMPACT_MAX_LAYERS];
  void* v[RB_COMPACT_MAX_LAYERS];
};
__global__ void compact_record_kernel(const __grid_constant__ KvLayers kv, int n_layers, int HK, int64_t s_head,
                                      int64_t s_slot, const int32_t* __restrict__ rec, int max_slots) {
  constexpr int kPieces = 128 * 2 / 16;  // 16-byte pieces of one bf16 row of 128
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (tid >= static_cast<int64_t>(n_layers) * 2 * HK * kPieces) return;
  const int n = rec[0], start = rec[3] + rec[2];
  const int piece = static_cast<int>(tid % kPieces);
  const int h = static_cast<int>((tid / kPieces) % HK);
  const int which = static_cast<int>((tid / (kPieces * HK)) % 2);
  const int layer = static_cast<int>(tid / (static_cast<int64_t>(kPieces) * HK * 2));
  uint8_t* base = static_cast<uint8_t*>(which ? kv.v[layer] : kv.k[layer]) + h * s_head * 2 + piece * 16;
  for (int i = 0; i < n; ++i) {
    const int src = start + rec[kAcceptHdr + i], dst = start + i;
    if (src == dst || src >= max_slots) continue;
    const uint4 val = *reinterpret_cast<const uint4*>(base + static_cast<int64_t>(src) * s_slot * 2);
    *reinterpret_cast<uint4*>(base + static_cast<int64_t>(dst) * s_slot * 2) = val;
  }
}

struct rb_engine {
  rb_model_config cfg;
  rb_model_weights w;
  std::vector<rb_layer_weights> layers;
  std::vector<void*> kc, vc;
  int dev = 0;
  int nsm = 148;
  // workspace carve-up
  StepParams* d_params = nullptr;
  int32_t *d_ids = nullptr, *d_parents = nullptr, *d_depths = nullptr, *d_chain = nullptr, *d_accept = nullptr;
  int64_t* d_out = nullptr;
  uint16_t *h = nullptr, *xn = nullptr, *qbuf = nullptr, *attn = nullptr, *act = nullptr;
  float *part = nullptr, *apart = nullptr, *logits = nullptr;
  unsigned long long* keys = nullptr;
  int max_chunks = 1;
  // tensor maps
  CUtensorMap m_xn, m_attn, m_act, m_lm;
  std::vector<CUtensorMap> m_qkv, m_o, m_gu, m_d, m_kc, m_vc;
  int bn_lm = 256;
  // host staging (a ring of pinned slots, so a host that enqueues many steps ahead,
  // a chunked prefill, waits only for the copy kStageSlots steps back) and graphs
  static constexpr int kStageSlots = 32;
  uint8_t* pinned = nullptr;
  size_t slot_bytes = 0;
  cudaEvent_t staged[kStageSlots] = {};
  bool staged_pending[kStageSlots] = {};
  int next_slot = 0;
  cudaStream_t cap = nullptr;
  std::map<int, cudaGraphExec_t> graphs;
  std::map<int, cudaGraph_t> graph_defs;
};

namespace {

constexpr int kQkvNT = 128;

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  size_t params, ids, parents, depths, chain, accept, out, keys, h, xn, qbuf, attn, act, part, apart, logits, total;
};

Layout layout_of(const rb_model_config& c) {
  Layout L{};
  const size_t R = static_cast<size_t>(c.max_rows);
  const int nsm = device_sm_count();
  const int nqkv = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
  const GemmShape s_qkv = gemm_plan(c.max_rows, nqkv, c.hidden, nsm);
  const GemmShape s_o = gemm_plan(c.max_rows, c.hidden, c.n_heads * c.head_dim, nsm);
  const GemmShape s_d = gemm_plan(c.max_rows, c.hidden, c.ffn, nsm);
  const GemmShape s_lm = gemm_plan(c.max_rows, c.vocab, c.hidden, nsm);
  size_t part_elems = static_cast<size_t>(s_qkv.splits) * nqkv;
  if (s_lm.splits > 1) part_elems = std::max(part_elems, static_cast<size_t>(s_lm.splits) * c.vocab);
  part_elems = std::max(part_elems, static_cast<size_t>(s_o.splits) * c.hidden);
  part_elems = std::max(part_elems, static_cast<size_t>(s_d.splits) * c.hidden);
  const int max_chunks = prefix_chunks_target(c.n_heads);
  size_t off = 0;
  auto take = [&](size_t bytes) { const size_t o = off; off = align256(off + bytes); return o; };
  L.params = take(sizeof(StepParams));
  L.ids = take(R * 4);
  L.parents = take(R * 4);
  L.depths = take(R * 4);
  L.chain = take(R * R * 4);
  L.accept = take((kAcceptHdr + 2 * R) * 4);
  L.out = take(R * 8);
  L.keys = take(R * 8);
  L.h = take(R * c.hidden * 2);
  L.xn = take(R * c.hidden * 2);
  L.qbuf = take(static_cast<size_t>(c.n_heads) * R * c.head_dim * 2);
  L.attn = take(R * c.n_heads * c.head_dim * 2);
  L.act = take(R * c.ffn * 2);
  L.part = take(part_elems * R * 4);
  L.apart = take(static_cast<size_t>(max_chunks) * c.n_heads * R * kPartStride * 4);
  L.logits = take(R * c.vocab * 4);
  L.total = off;
  return L;
}

int validate_cfg(const rb_model_config* c) {
  if (!c) return RB_ERR_INVALID_ARG;
  if (c->hidden <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv_heads <= 0 || c->ffn <= 0 ||
      c->vocab <= 0 || c->max_rows <= 0 || c->max_slots <= 0 || c->max_pos <= 0)
    return RB_ERR_INVALID_ARG;
  if (c->head_dim != 128 || c->n_heads % c->n_kv_heads != 0) return RB_ERR_UNSUPPORTED;
  if (c->hidden % 64 != 0 || c->ffn % 128 != 0 || c->vocab % 8 != 0) return RB_ERR_UNSUPPORTED;
  if (c->hidden > kMaxPerThread * 1024) return RB_ERR_UNSUPPORTED;
  if (c->max_rows > 1024 || c->n_layers > RB_COMPACT_MAX_LAYERS) return RB_ERR_CAPACITY;
  return RB_OK;
}

// Threads per row by N (the same choice as rmsnorm_kernel), elements per thread
// rounded up to a power of two for a statically indexed register array.
template <int NT, typename F>
int launch_norm_ept(int N, F&& f) {
  const int ept = (N + NT - 1) / NT;
  if (ept <= 1) return f(std::integral_constant<int, NT>{}, std::integral_constant<int, 1>{});
  if (ept <= 2) return f(std::integral_constant<int, NT>{}, std::integral_constant<int, 2>{});
  if (ept <= 4) return f(std::integral_constant<int, NT>{}, std::integral_constant<int, 4>{});
  if (ept <= 8) return f(std::integral_constant<int, NT>{}, std::integral_constant<int, 8>{});
  if (ept <= 16) return f(std::integral_constant<int, NT>{}, std::integral_constant<int, 16>{});
  if (ept <= 32) return f(std::integral_constant<int, NT>{}, std::integral_constant<int, 32>{});
  return RB_ERR_UNSUPPORTED;
}
template <typename F>
int launch_norm_nt(int N, F&& f) {
  if (N >= 2048) return launch_norm_ept<1024>(N, f);
  if (N >= 512) return launch_norm_ept<128>(N, f);
  return launch_norm_ept<32>(N, f);
}

#define RB_TRY(x)                     \
  do {                                \
    const int _st = (x);              \
    if (_st != RB_OK) return _st;     \
  } while (0)

int check_launch() { return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA; }

int launch_resid_norm(rb_engine* e, int splits, int rows, const void* w, cudaStream_t st) {
  const rb_model_config& c = e->cfg;
  return launch_norm_nt(c.hidden, [&](auto nt, auto ept) {
    constexpr int NT = decltype(nt)::value, EPT = decltype(ept)::value;
    if constexpr (NT == 1024) {
      constexpr int G4 = EPT < 4 ? 1 : EPT / 4;
      return launch_k(resid_norm_vec_kernel<G4>, dim3(rows), dim3(NT), 0, st, true,
                      static_cast<const StepParams*>(e->d_params), static_cast<const float*>(e->part), splits, rows,
                      e->h, static_cast<const uint16_t*>(w), e->xn, c.hidden, c.rms_eps);
    }
    auto go = [&](auto ms) {
      constexpr int MAXS = decltype(ms)::value;
      return launch_k(resid_norm_kernel<NT, EPT, MAXS>, dim3(rows), dim3(NT), 0, st, true,
                      static_cast<const StepParams*>(e->d_params), static_cast<const float*>(e->part), splits, rows,
                      e->h, static_cast<const uint16_t*>(w), e->xn, c.hidden, c.rms_eps);
    };
    if (splits <= 4) return go(std::integral_constant<int, 4>{});
    if (splits <= 8) return go(std::integral_constant<int, 8>{});
    if (splits <= 12) return go(std::integral_constant<int, 12>{});
    if (splits <= 16) return go(std::integral_constant<int, 16>{});
    return static_cast<int>(RB_ERR_UNSUPPORTED);
  });
}

// Enqueue one verify step for `rows` (bucketed) query rows on `st`.
int enqueue_step(rb_engine* e, int rows, cudaStream_t st) {
  const rb_model_config& c = e->cfg;
  const int H = c.n_heads, HK = c.n_kv_heads, D = c.head_dim;
  const int nqkv = (H + 2 * HK) * D;
  const int hid = c.hidden;
  const GemmShape s_qkv = gemm_plan(rows, nqkv, hid, e->nsm);
  const GemmShape s_o = gemm_plan(rows, hid, H * D, e->nsm);
  const GemmShape s_gu = gemm_plan(rows, 2 * c.ffn, hid, e->nsm, 256, 1);
  const GemmShape s_d = gemm_plan(rows, hid, c.ffn, e->nsm);
  const GemmShape s_lm = gemm_plan(rows, c.vocab, hid, e->nsm);
  if (s_lm.BN != e->bn_lm) return RB_ERR_INVALID_ARG;

  RB_TRY(launch_norm_nt(hid, [&](auto nt, auto ept) {
    constexpr int NT = decltype(nt)::value, EPT = decltype(ept)::value;
    constexpr int EV = NT == 1024 && EPT < 4 ? 4 : EPT;  // whole 4-column groups per thread
    return launch_k(embed_norm_kernel<NT, EV>, dim3(rows), dim3(NT), 0, st, true,
                    static_cast<const StepParams*>(e->d_params), static_cast<const int32_t*>(e->d_ids),
                    static_cast<const uint16_t*>(e->w.embed), static_cast<const uint16_t*>(e->layers[0].in_norm),
                    e->h, e->xn, hid, c.vocab, c.rms_eps, static_cast<const int32_t*>(e->d_parents),
                    static_cast<const int32_t*>(e->d_depths), e->d_chain, c.max_rows);
  }));
  for (int l = 0; l < c.n_layers; ++l) {
    const rb_layer_weights& lw = e->layers[l];
    GemmLaunch g{};
    g.w_tiled = 1;
    // q|k|v projection
    g.epi = kEpiPartial;
    g.partial = e->part;
    RB_TRY(gemm_launch_maps(s_qkv, e->m_xn, e->m_qkv[l], g, st, true));
    dim3 gq(rows, (H + 2 * HK + 3) / 4);
    RB_TRY(launch_k(qkv_finish_kernel, gq, dim3(kQkvNT), 0, st, true, static_cast<const StepParams*>(e->d_params),
                    static_cast<const int32_t*>(e->d_depths), static_cast<const float*>(e->part), s_qkv.splits, rows,
                    H, HK, static_cast<const uint16_t*>(lw.q_norm), static_cast<const uint16_t*>(lw.k_norm),
                    static_cast<const uint16_t*>(e->w.rope_cos), static_cast<const uint16_t*>(e->w.rope_sin),
                    c.max_pos, c.rms_eps, e->qbuf, static_cast<uint16_t*>(e->kc[l]),
                    static_cast<uint16_t*>(e->vc[l]), static_cast<int64_t>(c.max_slots) * D, c.max_slots));
    // attention over [prefix | committed | trie]
    AttnDev p{};
    p.H = H; p.M = rows; p.HK = HK; p.NP = 0; p.NN = 0;
    p.sp = e->d_params;
    p.depths = e->d_depths;
    p.chain = e->d_chain;
    p.chain_ld = c.max_rows;
    p.q = e->qbuf; p.sqh = static_cast<int64_t>(rows) * D; p.sqm = D;
    const int64_t sh = static_cast<int64_t>(c.max_slots) * D;
    p.kp = e->kc[l]; p.skph = sh; p.skpn = D;
    p.vp = e->vc[l]; p.svph = sh; p.svpn = D;
    // node slots start at the prompt length, which only the device knows:
    // kn/vn are set per step by the kernels from sp->prompt_len (see below).
    p.kn = nullptr; p.vn = nullptr; p.sknh = sh; p.sknn = D; p.svnh = sh; p.svnn = D;
    p.mask_kind = kMaskTrie;
    p.out = e->attn; p.soh = D; p.som = static_cast<int64_t>(H) * D;
    p.sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    CUtensorMap tq;  // q buffer is [H, rows, 128]: its head stride depends on the bucket
    RB_TRY(encode_heads_3d(&tq, e->qbuf, rows, H, D, static_cast<int64_t>(rows) * D));
    RB_TRY(attn_launch_engine(p, e->apart, e->max_chunks, tq, e->m_kc[l], e->m_vc[l], st));
    // o projection + residual + post-attention norm
    g.epi = kEpiPartial;
    RB_TRY(gemm_launch_maps(s_o, e->m_attn, e->m_o[l], g, st, true));
    RB_TRY(launch_resid_norm(e, s_o.splits, rows, lw.post_norm, st));
    // gate|up with the SiLU*mul epilogue
    GemmLaunch gu{};
    gu.w_tiled = 1;
    gu.epi = kEpiSiluMul;
    gu.out = e->act;
    gu.ldo = c.ffn;
    RB_TRY(gemm_launch_maps(s_gu, e->m_xn, e->m_gu[l], gu, st, true));
    // down + residual + next norm
    g.epi = kEpiPartial;
    RB_TRY(gemm_launch_maps(s_d, e->m_act, e->m_d[l], g, st, true));
    const void* next_norm = (l + 1 < c.n_layers) ? e->layers[l + 1].in_norm : e->w.final_norm;
    RB_TRY(launch_resid_norm(e, s_d.splits, rows, next_norm, st));
  }
  // lm_head (fp32 scores) with the greedy choice (acceptance.py:11-23) folded in;
  // the keys are zero on entry (zeroed at set-up, reset by the finalize kernel).
  GemmLaunch gl{};
  gl.w_tiled = 1;
  if (s_lm.splits == 1) {
    gl.epi = kEpiF32Argmax;
    gl.out = e->logits;
    gl.ldo = c.vocab;
    gl.keys = e->keys;
    gl.excl = &e->d_params->act_off;
    RB_TRY(gemm_launch_maps(s_lm, e->m_xn, e->m_lm, gl, st, true));
  } else {  // small vocabularies: split-K like rb_linear, fixed-order fp32 reduce
    gl.epi = kEpiPartial;
    gl.partial = e->part;
    RB_TRY(gemm_launch_maps(s_lm, e->m_xn, e->m_lm, gl, st, true));
    RB_TRY(splitk_reduce(e->part, s_lm.splits, rows, c.vocab, e->logits, c.vocab, 1, st));
    RB_TRY(launch_k(argmax_keys_kernel, dim3(8, rows), dim3(256), 0, st, false,
                    static_cast<const StepParams*>(e->d_params), static_cast<const float*>(e->logits),
                    static_cast<int64_t>(c.vocab), c.vocab, e->keys));
  }
  return launch_k(greedy_finalize_kernel, dim3((rows + 127) / 128), dim3(128), 0, st, true,
                  static_cast<const StepParams*>(e->d_params), e->keys, e->d_out, rows);
}

int bucket_of(int q) {
  int b = 1;
  while (b < q) b <<= 1;
  return b;
}

}  // namespace

extern "C" {

size_t rb_engine_workspace_bytes(const rb_model_config* cfg) {
  if (validate_cfg(cfg) != RB_OK) return 0;
  return layout_of(*cfg).total;
}

int rb_engine_create(const rb_model_config* cfg, const rb_model_weights* w, void* workspace, size_t ws_bytes,
                     rb_engine** out) {
  RB_TRY(validate_cfg(cfg));
  if (!w || !out || !w->layers || !w->k_cache || !w->v_cache || !w->embed || !w->final_norm || !w->lm_head ||
      !w->rope_cos || !w->rope_sin)
    return RB_ERR_INVALID_ARG;
  const Layout L = layout_of(*cfg);
  if (!workspace || ws_bytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255)) return RB_ERR_WORKSPACE;
  rb_engine* e = new rb_engine();
  e->cfg = *cfg;
  e->w = *w;
  e->layers.assign(w->layers, w->layers + cfg->n_layers);
  e->kc.assign(w->k_cache, w->k_cache + cfg->n_layers);
  e->vc.assign(w->v_cache, w->v_cache + cfg->n_layers);
  e->w.layers = nullptr;
  e->w.k_cache = e->w.v_cache = nullptr;
  cudaGetDevice(&e->dev);
  e->nsm = device_sm_count();
  uint8_t* base = static_cast<uint8_t*>(workspace);
  e->d_params = reinterpret_cast<StepParams*>(base + L.params);
  e->d_ids = reinterpret_cast<int32_t*>(base + L.ids);
  e->d_parents = reinterpret_cast<int32_t*>(base + L.parents);
  e->d_depths = reinterpret_cast<int32_t*>(base + L.depths);
  e->d_chain = reinterpret_cast<int32_t*>(base + L.chain);
  e->d_accept = reinterpret_cast<int32_t*>(base + L.accept);
  e->d_out = reinterpret_cast<int64_t*>(base + L.out);
  e->keys = reinterpret_cast<unsigned long long*>(base + L.keys);
  e->h = reinterpret_cast<uint16_t*>(base + L.h);
  e->xn = reinterpret_cast<uint16_t*>(base + L.xn);
  e->qbuf = reinterpret_cast<uint16_t*>(base + L.qbuf);
  e->attn = reinterpret_cast<uint16_t*>(base + L.attn);
  e->act = reinterpret_cast<uint16_t*>(base + L.act);
  e->part = reinterpret_cast<float*>(base + L.part);
  e->apart = reinterpret_cast<float*>(base + L.apart);
  e->logits = reinterpret_cast<float*>(base + L.logits);
  e->max_chunks = prefix_chunks_target(cfg->n_heads);

  const rb_model_config& c = *cfg;
  const int nqkv = (c.n_heads + 2 * c.n_kv_heads) * c.head_dim;
  int st = RB_OK;
  st |= gemm_encode_x(&e->m_xn, e->xn, c.max_rows, c.hidden, c.hidden);
  st |= gemm_encode_x(&e->m_attn, e->attn, c.max_rows, c.n_heads * c.head_dim, c.n_heads * c.head_dim);
  st |= gemm_encode_x(&e->m_act, e->act, c.max_rows, c.ffn, c.ffn);
  const GemmShape s_qkv = gemm_plan(1, nqkv, c.hidden, e->nsm);
  const GemmShape s_o = gemm_plan(1, c.hidden, c.n_heads * c.head_dim, e->nsm);
  const GemmShape s_d = gemm_plan(1, c.hidden, c.ffn, e->nsm);
  const GemmShape s_lm = gemm_plan(1, c.vocab, c.hidden, e->nsm);
  e->bn_lm = s_lm.BN;
  e->m_qkv.resize(c.n_layers);
  e->m_o.resize(c.n_layers);
  e->m_gu.resize(c.n_layers);
  e->m_d.resize(c.n_layers);
  e->m_kc.resize(c.n_layers);
  e->m_vc.resize(c.n_layers);
  for (int l = 0; l < c.n_layers && st == RB_OK; ++l) {
    const rb_layer_weights& lw = e->layers[l];
    if (!lw.wqkv || !lw.wo || !lw.wgu || !lw.wd || !lw.in_norm || !lw.post_norm || !lw.q_norm || !lw.k_norm ||
        !e->kc[l] || !e->vc[l]) {
      st = RB_ERR_INVALID_ARG;
      break;
    }
    st |= gemm_encode_w_packed(&e->m_qkv[l], lw.wqkv, nqkv, c.hidden, s_qkv.BN);
    st |= gemm_encode_w_packed(&e->m_o[l], lw.wo, c.hidden, c.n_heads * c.head_dim, s_o.BN);
    st |= gemm_encode_w_packed(&e->m_gu[l], lw.wgu, 2 * c.ffn, c.hidden, 256);
    st |= gemm_encode_w_packed(&e->m_d[l], lw.wd, c.hidden, c.ffn, s_d.BN);
    const int64_t sh = static_cast<int64_t>(c.max_slots) * c.head_dim;
    st |= encode_heads_3d(&e->m_kc[l], e->kc[l], c.max_slots, c.n_kv_heads, c.head_dim, sh);
    st |= encode_heads_3d(&e->m_vc[l], e->vc[l], c.max_slots, c.n_kv_heads, c.head_dim, sh);
  }
  if (st == RB_OK) st = gemm_encode_w_packed(&e->m_lm, w->lm_head, c.vocab, c.hidden, s_lm.BN);
  if (st != RB_OK) {
    delete e;
    return st != RB_ERR_INVALID_ARG ? RB_ERR_UNSUPPORTED : st;
  }
  if (cudaMemset(e->keys, 0, static_cast<size_t>(c.max_rows) * 8) != cudaSuccess) {
    delete e;
    return RB_ERR_CUDA;
  }
  e->slot_bytes = align256(sizeof(StepParams) + 3 * static_cast<size_t>(c.max_rows) * 4);
  bool ok = cudaMallocHost(&e->pinned, e->slot_bytes * rb_engine::kStageSlots) == cudaSuccess &&
            cudaStreamCreateWithFlags(&e->cap, cudaStreamNonBlocking) == cudaSuccess;
  for (int i = 0; ok && i < rb_engine::kStageSlots; ++i)
    ok = cudaEventCreateWithFlags(&e->staged[i], cudaEventDisableTiming) == cudaSuccess;
  if (!ok) {
    rb_engine_destroy(e);
    return RB_ERR_CUDA;
  }
  *out = e;
  return RB_OK;
}

int rb_engine_destroy(rb_engine* e) {
  if (!e) return RB_OK;
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : e->graph_defs) cudaGraphDestroy(kv.second);
  for (int i = 0; i < rb_engine::kStageSlots; ++i)
    if (e->staged[i]) cudaEventDestroy(e->staged[i]);
  if (e->cap) cudaStreamDestroy(e->cap);
  if (e->pinned) cudaFreeHost(e->pinned);
  delete e;
  return RB_OK;
}

int rb_engine_step(rb_engine* e, const rb_step_desc* d, void* stream) {
  if (!e || !d) return RB_ERR_INVALID_ARG;
  const rb_model_config& c = e->cfg;
  if (d->q <= 0 || d->base < 0 || d->prompt_len < 0 || !d->ids || !d->parents || !d->depths)
    return RB_ERR_INVALID_ARG;
  if (d->q > c.max_rows) return RB_ERR_CAPACITY;
  if (static_cast<int64_t>(d->prompt_len) + d->base + d->q > c.max_slots) return RB_ERR_CAPACITY;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  StepParams sp{};
  sp.q = d->q;
  sp.base = d->base;
  sp.prompt_len = d->prompt_len;
  sp.rope_delta = d->rope_delta;
  sp.act_off = d->act_off;
  sp.act_size = d->act_size;
  const size_t n4 = static_cast<size_t>(d->q) * 4;
  if (d->host_inputs) {
    // Validate the trie on the host (parents precede children, depth = parent + 1).
    for (int i = 0; i < d->q; ++i) {
      const int p = d->parents[i];
      if (p >= i || p < -1) return RB_ERR_INVALID_ARG;
      if (d->depths[i] != (p < 0 ? 0 : d->depths[p] + 1)) return RB_ERR_INVALID_ARG;
      if (d->ids[i] < 0 || d->ids[i] >= c.vocab) return RB_ERR_INVALID_ARG;
    }
  }
  const int slot = e->next_slot;
  e->next_slot = (slot + 1) % rb_engine::kStageSlots;
  if (e->staged_pending[slot]) {  // this slot's previous copy must have left the pinned buffer
    if (cudaEventSynchronize(e->staged[slot]) != cudaSuccess) return RB_ERR_CUDA;
    e->staged_pending[slot] = false;
  }
  uint8_t* p = e->pinned + static_cast<size_t>(slot) * e->slot_bytes;
  memcpy(p, &sp, sizeof(sp));
  if (cudaMemcpyAsync(e->d_params, p, sizeof(sp), cudaMemcpyHostToDevice, st) != cudaSuccess) return RB_ERR_CUDA;
  if (d->host_inputs) {
    // params, ids, parents, depths are laid out back to back in the workspace
    // only up to alignment, so copy each piece to its place.
    memcpy(p + sizeof(sp), d->ids, n4);
    memcpy(p + sizeof(sp) + n4, d->parents, n4);
    memcpy(p + sizeof(sp) + 2 * n4, d->depths, n4);
    if (cudaMemcpyAsync(e->d_ids, p + sizeof(sp), n4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_parents, p + sizeof(sp) + n4, n4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_depths, p + sizeof(sp) + 2 * n4, n4, cudaMemcpyHostToDevice, st) != cudaSuccess)
      return RB_ERR_CUDA;
  } else {
    if (cudaMemcpyAsync(e->d_ids, d->ids, n4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_parents, d->parents, n4, cudaMemcpyDeviceToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(e->d_depths, d->depths, n4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return RB_ERR_CUDA;
  }
  if (cudaEventRecord(e->staged[slot], st) != cudaSuccess) return RB_ERR_CUDA;
  e->staged_pending[slot] = true;
  const int rows = std::min(bucket_of(d->q), c.max_rows);  // workspace holds max_rows rows
  if (!d->use_graph) return enqueue_step(e, rows, st);
  auto it = e->graphs.find(rows);
  if (it == e->graphs.end()) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(e->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return RB_ERR_CUDA;
    const int r = enqueue_step(e, rows, e->cap);
    const cudaError_t ce = cudaStreamEndCapture(e->cap, &g);
    if (r != RB_OK) {
      if (g) cudaGraphDestroy(g);
      return r;
    }
    if (ce != cudaSuccess) return RB_ERR_CUDA;
    cudaGraphExec_t ge = nullptr;
    if (cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) {
      cudaGraphDestroy(g);
      return RB_ERR_CUDA;
    }
    e->graph_defs[rows] = g;
    it = e->graphs.emplace(rows, ge).first;
  }
  return cudaGraphLaunch(it->second, st) == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

int rb_engine_outputs(rb_engine* e, float** logits, int64_t** next_ids, void** hidden, void** kv_unused) {
  (void)kv_unused;
  if (!e) return RB_ERR_INVALID_ARG;
  if (logits) *logits = e->logits;
  if (next_ids) *next_ids = e->d_out;
  if (hidden) *hidden = e->h;
  return RB_OK;
}

int rb_engine_fetch_ids(rb_engine* e, int64_t* host, int n, void* stream) {
  if (!e || !host || n < 0 || n > e->cfg.max_rows) return RB_ERR_INVALID_ARG;
  if (n == 0) return RB_OK;
  return cudaMemcpyAsync(host, e->d_out, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToHost,
                         static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? RB_OK
             : RB_ERR_CUDA;
}

int rb_engine_compact(rb_engine* e, const int32_t* path, int n, int prompt_len, int base, void* stream) {
  if (!e || (n > 0 && !path) || n < 0 || prompt_len < 0 || base < 0) return RB_ERR_INVALID_ARG;
  if (n == 0) return RB_OK;
  if (n > RB_COMPACT_MAX_SLOTS) return RB_ERR_CAPACITY;
  std::vector<int32_t> src(n);
  for (int i = 0; i < n; ++i) {
    src[i] = prompt_len + base + path[i];
    if (src[i] >= e->cfg.max_slots) return RB_ERR_CAPACITY;
  }
  const rb_model_config& c = e->cfg;
  return compact_launch(e->kc.data(), e->vc.data(), c.n_layers, c.n_kv_heads, c.head_dim,
                        static_cast<int64_t>(c.max_slots) * c.head_dim, c.head_dim, 2, src.data(), n,
                        prompt_len + base, static_cast<cudaStream_t>(stream));
}

int rb_engine_accept(rb_engine* e, int first, int cap, int eos, void* stream) {
  if (!e || cap < 0) return RB_ERR_INVALID_ARG;
  const rb_model_config& c = e->cfg;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  accept_kernel<<<1, 1024, 0, st>>>(e->d_params, e->d_ids, e->d_parents, e->d_depths, e->d_out, first, cap, eos,
                                    c.max_rows, e->d_accept);
  if (cudaGetLastError() != cudaSuccess) return RB_ERR_CUDA;
  KvLayers kv{};
  for (int l = 0; l < c.n_layers; ++l) {
    kv.k[l] = e->kc[l];
    kv.v[l] = e->vc[l];
  }
  const int64_t total = static_cast<int64_t>(c.n_layers) * 2 * c.n_kv_heads * (128 * 2 / 16);
  compact_record_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(
      kv, c.n_layers, c.n_kv_heads, static_cast<int64_t>(c.max_slots) * c.head_dim, c.head_dim, e->d_accept,
      c.max_slots);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

int rb_engine_fetch_accept(rb_engine* e, int32_t* host, int n, void* stream) {
  if (!e || !host || n < 0 || n > e->cfg.max_rows) return RB_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t hdr = kAcceptHdr * 4, nb = static_cast<size_t>(n) * 4;
  if (cudaMemcpyAsync(host, e->d_accept, hdr, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      (n > 0 && (cudaMemcpyAsync(host + kAcceptHdr, e->d_accept + kAcceptHdr, nb, cudaMemcpyDeviceToHost, st) !=
                     cudaSuccess ||
                 cudaMemcpyAsync(host + kAcceptHdr + n, e->d_accept + kAcceptHdr + e->cfg.max_rows, nb,
                                 cudaMemcpyDeviceToHost, st) != cudaSuccess)))
    return RB_ERR_CUDA;
  return RB_OK;
}

}  // extern "C"
