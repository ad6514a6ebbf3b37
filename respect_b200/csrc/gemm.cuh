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
};

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
};

// Encodes the tensor maps and launches. Returns an rb_status code.
int gemm_launch(const GemmShape& s, const GemmLaunch& a, cudaStream_t stream);

// Same, with pre-encoded tensor maps (engine path: encoded once at set-up).
int gemm_launch_maps(const GemmShape& s, const CUtensorMap& mx, const CUtensorMap& mw,
                     const GemmLaunch& a, cudaStream_t stream);
int gemm_encode_x(CUtensorMap* m, const void* x, int M, int K, int64_t ldx);
int gemm_encode_w(CUtensorMap* m, const void* w, int N, int K, int64_t ldw, int BN);

// Sum split partials in ascending split order and store (bf16 or fp32).
int splitk_reduce(const float* partial, int splits, int M, int N, void* out, int64_t ldo,
                  int out_f32, cudaStream_t stream);

}  // namespace rb
