// Trie-verification attention: device parameter block and launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/respect_b200.h"

namespace rb {

// Prefix keys [0, NP) are reduced in chunks of prefix_chunk(NP, H) keys at
// absolute positions [c*C, (c+1)*C). The chunk size depends on the prefix
// length and the head count only (never on the number of query rows, the
// nodes or the device), so the trie and the 1-token AR steps over the same
// prefix split it identically. It aims at kChunkSlots / H chunks so that one
// 128-row tile of every head fills the GPU in one wave.
constexpr int kChunkSlots = 148;
constexpr int kMaxChunks = 16;
__host__ __device__ inline int prefix_chunks_target(int H) {
  const int t = kChunkSlots / (H > 0 ? H : 1);
  return t < 1 ? 1 : (t > kMaxChunks ? kMaxChunks : t);
}
__host__ __device__ inline int prefix_chunk(int NP, int H) {
  const int t = prefix_chunks_target(H);
  const int per = (NP + t - 1) / t;
  const int c = ((per + 127) / 128) * 128;
  return c < 128 ? 128 : c;
}
__host__ __device__ inline int prefix_nchunks(int NP, int H) {
  if (NP <= 0) return 0;
  const int c = prefix_chunk(NP, H);
  return (NP + c - 1) / c;
}
// Per (chunk, head, row) partial: acc[128], max (log2 domain), sum, 2 pad.
constexpr int kPartStride = 128 + 4;

// Step values an engine graph reads from device memory at run time, so that
// one captured graph serves every (rows <= bucket, committed, prompt length).
struct StepParams {
  int q;           // live query rows (trie nodes)
  int base;        // committed tokens after the prompt
  int prompt_len;  // PL: keys [0, PL) are the prefix
  int rope_delta;  // added to every rotary position (verify.py:31)
  int act_off, act_size;  // excluded vocabulary range of the greedy choice
  int pad[2];
};

// Node masking modes beyond the public rb_mask_kind values.
constexpr int kMaskTrie = 16;  // committed slots [0, base) then the row's ancestors, from chain[]

struct AttnDev {
  int H, M, HK, NP, NN;
  const StepParams* sp;       // non-null: q, base and NP come from device memory
  const int32_t* depths;      // kMaskTrie: depth of every node
  const int32_t* chain;       // kMaskTrie: row r's ancestors root first, chain[r * chain_ld + t], t <= depth
  int chain_ld;
  const void* q; int64_t sqh, sqm;
  const void* kp; int64_t skph, skpn;
  const void* vp; int64_t svph, svpn;
  const void* kn; int64_t sknh, sknn;
  const void* vn; int64_t svnh, svnn;
  const void* msk; int mask_kind; int64_t smm, smn;
  int causal_first;
  void* out; int64_t soh, som;
  float sm_scale;
};

size_t attn_workspace_bytes(int H, int M, int D, int NP);
int attn_validate(const rb_attn_args* a);
int attn_launch(const rb_attn_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
int attn_launch_engine(const AttnDev& p, float* part, int max_chunks, const CUtensorMap& tq,
                       const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream);
// 3-D tensor map of [heads, rows, 128] bf16 with 64 x 128 x 1 boxes (TMA, 128-byte swizzle).
int encode_heads_3d(CUtensorMap* m, const void* base, int rows, int heads, int64_t ld_row, int64_t ld_head);
int attn_prefix_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttnDev& p,
                          float* part, int nchunks, cudaStream_t stream, bool pdl);

}  // namespace rb
