// Launchers for the elementwise / per-row kernels (elementwise.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rb {

int rmsnorm_launch(const void* x, const void* w, void* y, int M, int N, float eps, int xdt, int wdt,
                   cudaStream_t s);
int rope_launch(const void* x, int64_t sxb, int64_t sxh, int64_t sxl, int64_t sxd, const void* c,
                const void* s, int64_t scb, int64_t scl, void* y, int B, int H, int L, int D, int xdt,
                int cdt, int ydt, cudaStream_t st);
int add_sq_launch(const void* r, const void* h, void* x, float* sq, int64_t n, int tr, int th, int tx,
                  cudaStream_t s);
int norm_apply_launch(const void* x, const float* var, const void* w, void* y, int64_t M, int N, float eps, int tx,
                      int tw, int ty, cudaStream_t s);
int silu_mul_launch(const void* g, const void* u, void* y, int64_t n, int dtype, cudaStream_t s);
int greedy_launch(const void* logits, int dt, int64_t ld, int M, int V, int off, int size, int64_t* out,
                  cudaStream_t s);
int compact_launch(void* const* k, void* const* v, int n_layers, int HK, int D, int64_t s_head,
                   int64_t s_slot, int elem_bytes, const int32_t* src, int n, int dst_start, cudaStream_t s);
int trie_node_mask_launch(const int32_t* parents, int q, int committed, int M, int NN, uint8_t* msk,
                          int64_t ld, cudaStream_t s);
int verify_mask_launch(const int32_t* parents, int q, int start, int width, void* m, cudaStream_t s);

}  // namespace rb
