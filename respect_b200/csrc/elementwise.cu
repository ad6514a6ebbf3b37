// Row-invariant RMSNorm, bit-exact RoPE and SiLU*mul, greedy argmax with the
// action-vocabulary mask, KV compaction and trie masks.
#include "common.cuh"
#include "elementwise.cuh"
#include "host_util.h"

namespace rb {

template <typename T> __device__ __forceinline__ float ld_f32(const T* p);
template <> __device__ __forceinline__ float ld_f32<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ld_f32<uint16_t>(const uint16_t* p) { return bf16_bits_to_f32(*p); }
template <typename T> __device__ __forceinline__ void st_f32(T* p, float v);
template <> __device__ __forceinline__ void st_f32<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st_f32<uint16_t>(uint16_t* p, float v) { *p = f32_to_bf16_bits(v); }
template <typename T> struct IsBF16 { static constexpr bool value = false; };
template <> struct IsBF16<uint16_t> { static constexpr bool value = true; };

// ------------------------------------------------------------------ RMSNorm
// One group of NT threads per row (respect/kernels/rmsnorm.py:12-22). Each
// thread sums a fixed subset of the row, then a fixed warp tree and a fixed
// cross-warp order: the row's bits never depend on the number of rows.
// Ownership: with VEC (NT = 1024, N % 4 == 0) thread t owns the 4-element
// groups 4(t + j NT) .. +3, summed j-major; otherwise the elements t + j NT.
// The engine's fused norms (embed / residual) use the same rule, so they stay
// bitwise equal to this operator. Rounding points follow PyTorch: upcast, mean
// of squares, rsqrt, downcast to the input dtype, multiply by the weight,
// downcast.
template <typename TX, typename TW, int NT, bool VEC>
__global__ void __launch_bounds__(NT >= 256 ? NT : 256) rmsnorm_kernel(const TX* __restrict__ x,
                                                                      const TW* __restrict__ w,
                                                                      TX* __restrict__ y, int M, int N, float eps) {
  constexpr int kRowsPerBlock = NT >= 256 ? 1 : 256 / NT;  // blocks of max(NT, 256) threads
  constexpr int kWarps = NT / 32;
  constexpr int kStep = VEC ? 4 * NT : NT;
  constexpr int kLanes = VEC ? 4 : 1;
  __shared__ float red[kRowsPerBlock][kWarps];
  const int sub = threadIdx.x / NT, t = threadIdx.x % NT;
  const int row = blockIdx.x * kRowsPerBlock + sub;
  const bool live = row < M;
  const TX* xr = x + static_cast<int64_t>(live ? row : 0) * N;
  const int first = VEC ? 4 * t : t;
  float ss = 0.f;
  if (live)
    for (int i = first; i < N; i += kStep) {
#pragma unroll
      for (int c = 0; c < kLanes; ++c) {
        const float v = ld_f32(xr + i + c);
        ss = fmaf(v, v, ss);
      }
    }
  ss = warp_sum(ss);
  ss = __shfl_sync(0xffffffffu, ss, 0);
  if ((t & 31) == 0) red[sub][t >> 5] = ss;
  __syncthreads();
  if (!live) return;
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) tot += red[sub][i];
  const float r = rsqrtf(tot / static_cast<float>(N) + eps);
  TX* yr = y + static_cast<int64_t>(row) * N;
  for (int i = t; i < N; i += NT) {
    float xh = ld_f32(xr + i) * r;
    if (IsBF16<TX>::value) xh = round_bf16(xh);
    st_f32(yr + i, ld_f32(w + i) * xh);
  }
}

template <typename TX, typename TW>
static int rmsnorm_t(const void* x, const void* w, void* y, int M, int N, float eps, cudaStream_t s) {
  const TX* xp = static_cast<const TX*>(x);
  const TW* wp = static_cast<const TW*>(w);
  TX* yp = static_cast<TX*>(y);
  if (M <= 0) return RB_OK;
  // Threads per row depend on N only.
  if (N >= 2048 && N % 4 == 0) {
    rmsnorm_kernel<TX, TW, 1024, true><<<M, 1024, 0, s>>>(xp, wp, yp, M, N, eps);
  } else if (N >= 2048) {
    rmsnorm_kernel<TX, TW, 1024, false><<<M, 1024, 0, s>>>(xp, wp, yp, M, N, eps);
  } else if (N >= 512) {
    rmsnorm_kernel<TX, TW, 128, false><<<(M + 1) / 2, 256, 0, s>>>(xp, wp, yp, M, N, eps);
  } else {
    rmsnorm_kernel<TX, TW, 32, false><<<(M + 7) / 8, 256, 0, s>>>(xp, wp, yp, M, N, eps);
  }
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

int rmsnorm_launch(const void* x, const void* w, void* y, int M, int N, float eps, int xdt, int wdt,
                   cudaStream_t s) {
  if (xdt == RB_BF16 && wdt == RB_BF16) return rmsnorm_t<uint16_t, uint16_t>(x, w, y, M, N, eps, s);
  if (xdt == RB_BF16 && wdt == RB_F32) return rmsnorm_t<uint16_t, float>(x, w, y, M, N, eps, s);
  if (xdt == RB_F32 && wdt == RB_F32) return rmsnorm_t<float, float>(x, w, y, M, N, eps, s);
  if (xdt == RB_F32 && wdt == RB_BF16) return rmsnorm_t<float, uint16_t>(x, w, y, M, N, eps, s);
  return RB_ERR_UNSUPPORTED;
}

// ------------------------------------------------------------------ RoPE
// y = x*cos + rotate_half(x)*sin, every product and the sum rounded to bf16
// when ROUND (bf16 output), no FMA contraction (respect/system/fused.py:45-64).
template <typename TX, typename TC, typename TY, bool ROUND>
__global__ void rope_kernel(const TX* __restrict__ x, int64_t sxb, int64_t sxh, int64_t sxl, int64_t sxd,
                            const TC* __restrict__ cs, const TC* __restrict__ sn, int64_t scb, int64_t scl,
                            TY* __restrict__ y, int H, int L, int D, int64_t total_rows) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= total_rows) return;
  const int l = static_cast<int>(row % L);
  const int h = static_cast<int>((row / L) % H);
  const int b = static_cast<int>(row / (static_cast<int64_t>(L) * H));
  const int half = D / 2;
  const TX* xb = x + b * sxb + h * sxh + l * sxl;
  const TC* cb = cs + b * scb + l * scl;
  const TC* sb = sn + b * scb + l * scl;
  TY* yb = y + row * D;
  for (int d = threadIdx.x & 31; d < D; d += 32) {
    const float xv = ld_f32(xb + d * sxd);
    const int dr = d < half ? d + half : d - half;
    float xr = ld_f32(xb + dr * sxd);
    xr = d < half ? -xr : xr;
    const float c = ld_f32(cb + d), s = ld_f32(sb + d);
    float a = __fmul_rn(xv, c);
    float r = __fmul_rn(xr, s);
    if (ROUND) { a = round_bf16(a); r = round_bf16(r); }
    float o = __fadd_rn(a, r);
    if (ROUND) o = round_bf16(o);
    st_f32(yb + d, o);
  }
}

template <typename TX, typename TC, typename TY, bool ROUND>
static int rope_t(const void* x, int64_t sxb, int64_t sxh, int64_t sxl, int64_t sxd, const void* c,
                  const void* s, int64_t scb, int64_t scl, void* y, int B, int H, int L, int D,
                  cudaStream_t st) {
  const int64_t rows = static_cast<int64_t>(B) * H * L;
  if (rows == 0) return RB_OK;
  const int64_t blocks = (rows + 7) / 8;
  if (blocks > 0x7fffffff) return RB_ERR_CAPACITY;
  rope_kernel<TX, TC, TY, ROUND><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const TX*>(x), sxb, sxh, sxl, sxd, static_cast<const TC*>(c), static_cast<const TC*>(s),
      scb, scl, static_cast<TY*>(y), H, L, D, rows);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

int rope_launch(const void* x, int64_t sxb, int64_t sxh, int64_t sxl, int64_t sxd, const void* c,
                const void* s, int64_t scb, int64_t scl, void* y, int B, int H, int L, int D, int xdt,
                int cdt, int ydt, cudaStream_t st) {
  // Output dtype is torch.promote_types(x, cos): bf16 only when both are bf16.
  const int want = (xdt == RB_BF16 && cdt == RB_BF16) ? RB_BF16 : RB_F32;
  if (ydt != want) return RB_ERR_INVALID_ARG;
  if (xdt == RB_BF16 && cdt == RB_BF16)
    return rope_t<uint16_t, uint16_t, uint16_t, true>(x, sxb, sxh, sxl, sxd, c, s, scb, scl, y, B, H, L, D, st);
  if (xdt == RB_F32 && cdt == RB_F32)
    return rope_t<float, float, float, false>(x, sxb, sxh, sxl, sxd, c, s, scb, scl, y, B, H, L, D, st);
  if (xdt == RB_BF16 && cdt == RB_F32)
    return rope_t<uint16_t, float, float, false>(x, sxb, sxh, sxl, sxd, c, s, scb, scl, y, B, H, L, D, st);
  if (xdt == RB_F32 && cdt == RB_BF16)
    return rope_t<float, uint16_t, float, false>(x, sxb, sxh, sxl, sxd, c, s, scb, scl, y, B, H, L, D, st);
  return RB_ERR_UNSUPPORTED;
}

// ------------------------------------------------------------------ SiLU*mul
// y = bf16(bf16(g / (1 + exp(-g))) * u) (respect/system/fused.py:106-113);
// expf and the IEEE divide are CUDA's own.
__global__ void silu_mul_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                                uint16_t* __restrict__ y, int64_t n) {
  const int64_t i0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i0 + 8 <= n) {
    const uint4 gv = *reinterpret_cast<const uint4*>(g + i0);
    const uint4 uv = *reinterpret_cast<const uint4*>(u + i0);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&uv);
    uint4 ov;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&ov);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float r[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gf = bf16_bits_to_f32(static_cast<uint16_t>(gw[k] >> (16 * e)));
        const float uf = bf16_bits_to_f32(static_cast<uint16_t>(uw[k] >> (16 * e)));
        const float s = round_bf16(gf / (1.0f + expf(-gf)));
        r[e] = __fmul_rn(s, uf);
      }
      ow[k] = pack_bf16x2(r[0], r[1]);
    }
    *reinterpret_cast<uint4*>(y + i0) = ov;
  } else {
    for (int64_t i = i0; i < n; ++i) {
      const float gf = bf16_bits_to_f32(g[i]);
      const float uf = bf16_bits_to_f32(u[i]);
      const float s = round_bf16(gf / (1.0f + expf(-gf)));
      y[i] = f32_to_bf16_bits(__fmul_rn(s, uf));
    }
  }
}

// fp32 inputs: silu in fp32, then the product in fp32 (PyTorch eager
// `silu(g) * u`); the reference routes this dtype to eager (fused.py:117-118).
__global__ void silu_mul_f32_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                    float* __restrict__ y, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    const float gf = g[i];
    y[i] = __fmul_rn(gf / (1.0f + expf(-gf)), u[i]);
  }
}

// ------------------------------------------------------------------ prefill norms
// respect/system/fused.py:126-194: the pieces of an eager RMSNorm (with the
// residual add before it) whose bits PyTorch fixes elementwise, around the row
// mean that PyTorch itself computes. add_sq: x = r + h in the promoted dtype
// (rounded to bf16 when that is bf16), sq = x * x in fp32; with h == nullptr,
// sq = r * r only. norm_apply: y = w * to_x_dtype(x * rsqrt(var + eps)) with
// the output in promote(w, x) (rounded to bf16 when that is bf16).
template <typename T>
__device__ __forceinline__ float ld_f(const void* p, int64_t i) {
  if constexpr (sizeof(T) == 2) return bf16_bits_to_f32(static_cast<const uint16_t*>(p)[i]);
  else return static_cast<const float*>(p)[i];
}
template <typename T>
__device__ __forceinline__ void st_f(void* p, int64_t i, float v) {
  if constexpr (sizeof(T) == 2) static_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(v);
  else static_cast<float*>(p)[i] = v;
}

template <typename TR, typename TH, typename TX>
__global__ void add_sq_kernel(const void* __restrict__ r, const void* __restrict__ h, void* __restrict__ x,
                              float* __restrict__ sq, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v = ld_f<TR>(r, i);
    if (h) {
      v = __fadd_rn(v, ld_f<TH>(h, i));
      if constexpr (sizeof(TX) == 2) v = round_bf16(v);
      st_f<TX>(x, i, v);
    }
    sq[i] = __fmul_rn(v, v);
  }
}

template <typename TX, typename TW, typename TY>
__global__ void norm_apply_kernel(const void* __restrict__ x, const float* __restrict__ var, const void* __restrict__ w,
                                  void* __restrict__ y, int64_t M, int N, float eps) {
  const int64_t n = M * N;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / N;
    const int col = static_cast<int>(i - row * N);
    const float rs = rsqrtf(__fadd_rn(var[row], eps));
    float xh = __fmul_rn(ld_f<TX>(x, i), rs);
    if constexpr (sizeof(TX) == 2) xh = round_bf16(xh);
    float v = __fmul_rn(ld_f<TW>(w, col), xh);
    if constexpr (sizeof(TY) == 2) v = round_bf16(v);
    st_f<TY>(y, i, v);
  }
}

static unsigned ew_blocks(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 148 * 32 ? (b < 1 ? 1 : b) : 148 * 32);
}

int add_sq_launch(const void* r, const void* h, void* x, float* sq, int64_t n, int tr, int th, int tx,
                  cudaStream_t s) {
  if (n <= 0) return RB_OK;
  const unsigned g = ew_blocks(n);
  // promote(r, h): bf16 only when both are bf16
  const int want = h ? ((tr == RB_BF16 && th == RB_BF16) ? RB_BF16 : RB_F32) : tr;
  if (h && tx != want) return RB_ERR_UNSUPPORTED;
  if (!h) {
    if (tr == RB_BF16) add_sq_kernel<uint16_t, uint16_t, uint16_t><<<g, 256, 0, s>>>(r, nullptr, nullptr, sq, n);
    else add_sq_kernel<float, float, float><<<g, 256, 0, s>>>(r, nullptr, nullptr, sq, n);
  } else if (tr == RB_BF16 && th == RB_BF16) {
    add_sq_kernel<uint16_t, uint16_t, uint16_t><<<g, 256, 0, s>>>(r, h, x, sq, n);
  } else if (tr == RB_BF16) {
    add_sq_kernel<uint16_t, float, float><<<g, 256, 0, s>>>(r, h, x, sq, n);
  } else if (th == RB_BF16) {
    add_sq_kernel<float, uint16_t, float><<<g, 256, 0, s>>>(r, h, x, sq, n);
  } else {
    add_sq_kernel<float, float, float><<<g, 256, 0, s>>>(r, h, x, sq, n);
  }
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

int norm_apply_launch(const void* x, const float* var, const void* w, void* y, int64_t M, int N, float eps, int tx,
                      int tw, int ty, cudaStream_t s) {
  if (M <= 0) return RB_OK;
  const int want = (tx == RB_BF16 && tw == RB_BF16) ? RB_BF16 : RB_F32;
  if (ty != want) return RB_ERR_UNSUPPORTED;
  const unsigned g = ew_blocks(M * N);
#define RB_NORM_APPLY(A, B, C) norm_apply_kernel<A, B, C><<<g, 256, 0, s>>>(x, var, w, y, M, N, eps)
  if (tx == RB_BF16 && tw == RB_BF16) RB_NORM_APPLY(uint16_t, uint16_t, uint16_t);
  else if (tx == RB_BF16) RB_NORM_APPLY(uint16_t, float, float);
  else if (tw == RB_BF16) RB_NORM_APPLY(float, uint16_t, float);
  else RB_NORM_APPLY(float, float, float);
#undef RB_NORM_APPLY
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

int silu_mul_launch(const void* g, const void* u, void* y, int64_t n, int dtype, cudaStream_t s) {
  if (n <= 0) return RB_OK;
  if (dtype == RB_F32) {
    const int64_t blocks = (n + 255) / 256;
    if (blocks > 0x7fffffff) return RB_ERR_CAPACITY;
    silu_mul_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const float*>(g), static_cast<const float*>(u), static_cast<float*>(y), n);
    return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
  }
  if (dtype != RB_BF16) return RB_ERR_UNSUPPORTED;
  if (!aligned16(g) || !aligned16(u) || !aligned16(y)) return RB_ERR_UNSUPPORTED;
  const int64_t threads = (n + 7) / 8;
  const int64_t blocks = (threads + 255) / 256;
  if (blocks > 0x7fffffff) return RB_ERR_CAPACITY;
  silu_mul_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      static_cast<const uint16_t*>(g), static_cast<const uint16_t*>(u), static_cast<uint16_t*>(y), n);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

// ------------------------------------------------------------------ greedy token
// Row argmax with [offset, offset+size) excluded (acceptance.py:11-23). NaN
// counts as the largest value (torch.argmax); ties keep the lowest index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn != bn) return vn;
  if (vn) return i < bi;
  return v > bv || (v == bv && i < bi);
}

template <typename T>
__global__ void greedy_kernel(const T* __restrict__ logits, int64_t ld, int V, int off, int size,
                              int64_t* __restrict__ out) {
  const int row = blockIdx.x;
  const T* r = logits + static_cast<int64_t>(row) * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    if (i >= off && i < off + size) continue;
    const float v = ld_f32(r + i);
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    // A row whose every entry is excluded (or -inf) reports index 0, as argmax does.
    out[row] = (bi == 0x7fffffff) ? 0 : bi;
  }
}

int greedy_launch(const void* logits, int dt, int64_t ld, int M, int V, int off, int size, int64_t* out,
                  cudaStream_t s) {
  if (M <= 0) return RB_OK;
  if (dt == RB_F32) greedy_kernel<float><<<M, 1024, 0, s>>>(static_cast<const float*>(logits), ld, V, off, size, out);
  else if (dt == RB_BF16) greedy_kernel<uint16_t><<<M, 1024, 0, s>>>(static_cast<const uint16_t*>(logits), ld, V, off, size, out);
  else return RB_ERR_UNSUPPORTED;
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

// ------------------------------------------------------------------ compact
// One thread per (layer, K|V, head, 16-byte piece of a slot row). Each thread
// walks the path in ascending order: dst_start+i <= src[i] and src is
// increasing, so no slot is overwritten before it is read
// (respect/decoding/kv_buffer.py:93-104 gathers then scatters; the order here
// gives the same result without a temporary).
struct CompactParams {
  void* k[RB_COMPACT_MAX_LAYERS];
  void* v[RB_COMPACT_MAX_LAYERS];
  int32_t src[RB_COMPACT_MAX_SLOTS];
};

__global__ void compact_kernel(const __grid_constant__ CompactParams p, int n_layers, int HK,
                               int pieces, int64_t s_head, int64_t s_slot, int elem_bytes, int n,
                               int dst_start) {
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = static_cast<int64_t>(n_layers) * 2 * HK * pieces;
  if (tid >= total) return;
  const int piece = static_cast<int>(tid % pieces);
  const int h = static_cast<int>((tid / pieces) % HK);
  const int kv = static_cast<int>((tid / (static_cast<int64_t>(pieces) * HK)) % 2);
  const int layer = static_cast<int>(tid / (static_cast<int64_t>(pieces) * HK * 2));
  uint8_t* base = static_cast<uint8_t*>(kv ? p.v[layer] : p.k[layer]) + h * s_head * elem_bytes + piece * 16;
  for (int i = 0; i < n; ++i) {
    const int src = p.src[i], dst = dst_start + i;
    if (src == dst) continue;
    const uint4 val = *reinterpret_cast<const uint4*>(base + static_cast<int64_t>(src) * s_slot * elem_bytes);
    *reinterpret_cast<uint4*>(base + static_cast<int64_t>(dst) * s_slot * elem_bytes) = val;
  }
}

int compact_launch(void* const* k, void* const* v, int n_layers, int HK, int D, int64_t s_head,
                   int64_t s_slot, int elem_bytes, const int32_t* src, int n, int dst_start, cudaStream_t s) {
  if (n <= 0) return RB_OK;
  if (n_layers <= 0 || n_layers > RB_COMPACT_MAX_LAYERS || n > RB_COMPACT_MAX_SLOTS) return RB_ERR_CAPACITY;
  if ((D * elem_bytes) % 16 != 0 || (s_head * elem_bytes) % 16 != 0 || (s_slot * elem_bytes) % 16 != 0)
    return RB_ERR_UNSUPPORTED;
  CompactParams p;
  bool moves = false;
  for (int i = 0; i < n; ++i) {
    if (src[i] < dst_start + i || (i > 0 && src[i] <= src[i - 1])) return RB_ERR_INVALID_ARG;
    p.src[i] = src[i];
    moves |= src[i] != dst_start + i;
  }
  if (!moves) return RB_OK;  // same early exit as the reference (torch.equal(src, dst))
  for (int l = 0; l < n_layers; ++l) {
    if (!k[l] || !v[l] || !aligned16(k[l]) || !aligned16(v[l])) return RB_ERR_INVALID_ARG;
    p.k[l] = k[l];
    p.v[l] = v[l];
  }
  const int pieces = D * elem_bytes / 16;
  const int64_t total = static_cast<int64_t>(n_layers) * 2 * HK * pieces;
  compact_kernel<<<static_cast<unsigned>((total + 127) / 128), 128, 0, s>>>(p, n_layers, HK, pieces, s_head,
                                                                           s_slot, elem_bytes, n, dst_start);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

// ------------------------------------------------------------------ trie masks
// j is an ancestor-or-self of i iff walking i's parent chain reaches j.
// Parents precede children (trie.py:31-48), so the walk strictly decreases;
// a malformed parent (>= its child) stops the walk.
__device__ __forceinline__ bool is_ancestor(const int32_t* __restrict__ parents, int i, int j) {
  int a = i;
  while (a > j) {
    const int p = parents[a];
    if (p >= a) return false;
    a = p;
  }
  return a == j;
}

__global__ void trie_node_mask_kernel(const int32_t* __restrict__ parents, int q, int committed, int NN,
                                      uint8_t* __restrict__ msk, int64_t ld) {
  const int row = blockIdx.x;
  uint8_t* r = msk + static_cast<int64_t>(row) * ld;
  for (int j = threadIdx.x; j < NN; j += blockDim.x) {
    uint8_t v = 0;
    if (row < q) {
      if (j < committed) v = 1;
      else if (j < committed + q) v = is_ancestor(parents, row, j - committed) ? 1 : 0;
    } else {
      v = (j == 0) ? 1 : 0;  // padding rows open slot 0 (dispatch.py:115)
    }
    r[j] = v;
  }
}

int trie_node_mask_launch(const int32_t* parents, int q, int committed, int M, int NN, uint8_t* msk,
                          int64_t ld, cudaStream_t s) {
  if (M <= 0 || NN <= 0) return RB_OK;
  trie_node_mask_kernel<<<M, 256, 0, s>>>(parents, q, committed, NN, msk, ld);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

__global__ void verify_mask_kernel(const int32_t* __restrict__ parents, int q, int start, int width,
                                   uint16_t* __restrict__ m) {
  const int row = blockIdx.x;
  uint16_t* r = m + static_cast<int64_t>(row) * width;
  constexpr uint16_t kZero = 0x0000, kLowest = 0xFF7F;  // bf16 0 and torch.finfo(bf16).min
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    uint16_t v = kLowest;
    if (c < start) v = kZero;
    else if (c < start + q && is_ancestor(parents, row, c - start)) v = kZero;
    r[c] = v;
  }
}

int verify_mask_launch(const int32_t* parents, int q, int start, int width, void* m, cudaStream_t s) {
  if (q <= 0 || width <= 0) return RB_OK;
  verify_mask_kernel<<<q, 256, 0, s>>>(parents, q, start, width, static_cast<uint16_t*>(m));
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

}  // namespace rb
