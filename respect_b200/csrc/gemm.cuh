// Row-count-invariant weight-streaming GEMM for sm_100a.
//
//   C[m, n] = sum_k X[m, k] * W[n, k]        X: [M, K] bf16, W: [N, K] bf16
//
// Each CTA owns one BN-wide slab of weight rows (the MMA N side), one group of
// 128-row token tiles (the MMA M side, zero-padded by TMA) and one K range.
// Every output element is produced by the same sequence of
// tcgen05.mma.kind::f16 instructions (M=128, N=BN, K=16) over K in ascending
// order, whatever M is; the K split S depends on (N, K) only and the split
// partials are summed in ascending split order. A row therefore gives the same
// bits whether it is computed alone or with other rows, which is the property
// respect/kernels/gemm.py:1-5 states for the reference's Triton GEMM.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace rb {

enum GemmEpilogue : int {
  kEpiStoreBF16 = 0,  // out[m, n] = bf16(acc)
  kEpiStoreF32 = 1,   // out[m, n] = acc (lm_head scores)
  kEpiSiluMul = 2,    // W rows interleaved per BN block (gate | up): out[m, j] = bf16(bf16(silu(bf16 g)) * bf16 u)
  kEpiPartial = 3,    // partial[s, m, n] = acc (fp32, split-K)
  kEpiF32Argmax = 4,  // kEpiStoreF32 + per-row greedy choice folded into keys[m] by atomicMax
};

// Order-preserving 64-bit key of (value, index): larger value first, then the
// lower index; NaN above every number (torch.argmax). max() over keys is
// associative and commutative, so the choice does not depend on tile order.
__host__ __device__ inline unsigned long long argmax_key(float v, int idx) {
  unsigned int u;
  if (v != v) {
    u = 0xFFFFFFFFu;
  } else {
    if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal: one key
#ifdef __CUDA_ARCH__
    u = __float_as_uint(v);
#else
    union { float f; unsigned int i; } c{v};
    u = c.i;
#endif
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  return (static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - static_cast<unsigned int>(idx));
}

struct GemmShape {
  int M, N, K;
  int BN;        // weight rows per CTA tile
  int mt;        // 128-row token tiles per CTA (1 or 2)
  int splits;    // K splits
  int n_tiles, m_groups, k_chunks;
};

// Split / tile choice. Depends on N and K (never on M) so that row results are
// independent of the number of rows in a call.
GemmShape gemm_plan(int M, int N, int K, int num_sms, int force_bn = 0, int force_splits = 0);

struct GemmLaunch {
  const void* x; int64_t ldx;   // bf16 [M, K]
  const void* w; int64_t ldw;   // bf16 [N, K]
  void* out; int64_t ldo;       // epilogue output
  float* partial;               // [splits, M, N] fp32 (kEpiPartial)
  int epi;
  unsigned long long* keys;     // kEpiF32Argmax: [M] per-row keys (caller zeroes them)
  const int* excl;              // kEpiF32Argmax: {offset, size} of the excluded column range (device)
  int w_tiled;                  // w is packed (gemm_pack_weight) and its map from gemm_encode_w_packed
};

// Encodes the tensor maps and launches. Returns an rb_status code.
int gemm_launch(const GemmShape& s, const GemmLaunch& a, cudaStream_t stream);

// Same, with pre-encoded tensor maps (engine path: encoded once at set-up).
// pdl: launch with programmatic stream serialization (weight prefetch overlaps
// the previous kernel; see pdl_wait in common.cuh).
int gemm_launch_maps(const GemmShape& s, const CUtensorMap& mx, const CUtensorMap& mw,
                     const GemmLaunch& a, cudaStream_t stream, bool pdl = false);
int gemm_encode_x(CUtensorMap* m, const void* x, int M, int K, int64_t ldx);
int gemm_encode_w(CUtensorMap* m, const void* w, int N, int K, int64_t ldw, int BN);

// Packed weights: [ceil(N/BN)][ceil(K/64)][BN][64] bf16, zero padded, so each
// pipeline stage streams one contiguous BN x 128-byte block. The MMA sequence
// per output element is the same as with the row-major layout.
size_t gemm_packed_elems(int N, int K, int BN);
int gemm_encode_w_packed(CUtensorMap* m, const void* wp, int N, int K, int BN);
int gemm_pack_weight(const void* w, int64_t ldw, int N, int K, int BN, void* out, cudaStream_t st);

// Sum split partials in ascending split order and store (bf16 or fp32).
int splitk_reduce(const float* partial, int splits, int M, int N, void* out, int64_t ldo,
                  int out_f32, cudaStream_t stream);

}  // namespace rb
