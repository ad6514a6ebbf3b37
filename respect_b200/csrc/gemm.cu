// Row-count-invariant weight-streaming GEMM (tcgen05 + TMA, sm_100a).
// Follows the contract of respect/kernels/gemm.py:11-41: fixed K order, fp32
// accumulation, bf16 or fp32 output, bias handled by the caller.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "host_util.h"

namespace rb {

constexpr int kBK = 64;                          // K elements per stage: one 128-byte swizzle row
constexpr int kTileM = 128;                      // token rows per MMA (M side)
constexpr int kXTileBytes = kTileM * kBK * 2;    // 16 KB
constexpr int kSmemLimit = 232448;               // 227 KB dynamic shared memory per CTA

__host__ __device__ constexpr int pow2_cols(int c) {
  return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512;
}

// Shared memory: a ring of weight tiles (BN x 64, the DRAM stream, as deep as
// fits, at most WMAX) and a short ring of token tiles (MT x 128 x 64, L2-resident).
template <int BN, int MT, int WMAX = 12>
struct GemmCfg {
  static constexpr int kWTileBytes = BN * kBK * 2;
  static constexpr int kXStageBytes = MT * kXTileBytes;
  // Two token tiles per stage (256 rows) take as long in the tensor pipe as a
  // weight tile takes to arrive; a third token stage keeps their L2 round trip
  // (issued only when a stage is released) off the MMA's path.
  // 128-wide weight tiles (the short q|k|v and o projections) run their main
  // loop only once the previous kernel ends, with most of their weights already
  // in the ring: four token stages keep the token tiles' L2 round trips apart.
  static constexpr int kXStages = MT == 2 ? 3 : (BN <= 128 ? 4 : 2);
  static constexpr int kWStagesRaw = (kSmemLimit - 1024 - 256 - kXStages * kXStageBytes) / kWTileBytes;
  static constexpr int kWStages = kWStagesRaw > WMAX ? WMAX : kWStagesRaw;
  static constexpr int kWOff = 0;
  static constexpr int kXOff = kWStages * kWTileBytes;
  static constexpr int kBarOff = kXOff + kXStages * kXStageBytes;
  static constexpr int kAccStride = pow2_cols(BN);  // TMEM columns between token-tile accumulators
  static constexpr int kTmemCols = MT * kAccStride;
  static constexpr int kSmemBytes = 1024 + kBarOff + 256;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 is 16..256 step 16");
  static_assert(MT * pow2_cols(BN) <= 512, "TMEM holds 512 fp32 columns");
  static_assert(kWStages >= 3, "weight ring needs three stages");
  static_assert(kWTileBytes % 1024 == 0 && kXTileBytes % 1024 == 0, "swizzle atoms are 1024-byte aligned");
  static_assert(kSmemBytes <= kSmemLimit, "shared memory budget");
  static_assert((2 * kWStages + 2 * kXStages + 1) * 8 + 4 <= 256, "barriers and TMEM slot fit their 256 bytes");
};

// Output element size of an epilogue, and the row width in bytes of the
// shared-memory boxes the staged epilogue writes with TMA (0: not staged):
// 128-byte rows where a tile's output is a whole number of them, else 64.
// Staged: the split-K partials and the bf16 outputs, whose single-wave grids
// finish on their last CTA's stores. The fp32 outputs (the many-wave vocabulary
// projection) keep the direct per-thread stores, which the CTA does not wait
// for before it exits (measured: staging made the lm_head 4% slower).
__host__ __device__ constexpr int gemm_out_elem_bytes(int epi) {
  return (epi == kEpiStoreBF16 || epi == kEpiSiluMul) ? 2 : 4;
}
__host__ __device__ constexpr int gemm_stage_row_bytes(int epi, int bn) {
  return (epi == kEpiStoreF32 || epi == kEpiF32Argmax) ? 0
         : ((epi == kEpiSiluMul ? bn / 2 : bn) * gemm_out_elem_bytes(epi)) % 128 == 0 ? 128
         : ((epi == kEpiSiluMul ? bn / 2 : bn) * gemm_out_elem_bytes(epi)) % 64 == 0 ? 64
                                                                                     : 0;
}

// Weight-ring cap by epilogue. The fp32 outputs are the vocabulary projection,
// whose grid runs several CTAs per SM one after another: with three weight
// stages a CTA needs 111 KB of shared memory (BN = 208), so two share an SM and
// one's prologue and epilogue overlap the other's weight stream. The
// single-wave grids, and CTAs with two token tiles (which do not fit twice
// anyway), keep the deep ring.
__host__ __device__ constexpr int gemm_w_stage_cap(int epi, int mt) {
  return (mt == 1 && (epi == kEpiStoreF32 || epi == kEpiF32Argmax)) ? 3 : 12;
}

struct GemmKernelArgs {
  int M, N, K;
  int k_chunks, splits;
  int w_tiled;  // weights packed as [n_tile][k_chunk][BN][64] (gemm_pack_weight)

  void* out;
  int64_t ldo;
  float* partial;
  unsigned long long* keys;
  const int* excl;
  int tma_out;  // epilogue stages the tile in shared memory and writes it with TMA stores (tmo)
};

template <int EPI>
__device__ __forceinline__ void epi_store16_impl(const GemmKernelArgs& a, int m, int n0, int split,
                                            const float (&v)[16]) {
  if (EPI == kEpiStoreBF16) {
    uint16_t* o = static_cast<uint16_t*>(a.out) + static_cast<int64_t>(m) * a.ldo + n0;
    if (n0 + 16 <= a.N && (a.ldo & 7) == 0) {
      uint4 p0, p1;
      p0.x = pack_bf16x2(v[0], v[1]);   p0.y = pack_bf16x2(v[2], v[3]);
      p0.z = pack_bf16x2(v[4], v[5]);   p0.w = pack_bf16x2(v[6], v[7]);
      p1.x = pack_bf16x2(v[8], v[9]);   p1.y = pack_bf16x2(v[10], v[11]);
      p1.z = pack_bf16x2(v[12], v[13]); p1.w = pack_bf16x2(v[14], v[15]);
      reinterpret_cast<uint4*>(o)[0] = p0;
      reinterpret_cast<uint4*>(o)[1] = p1;
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n0 + i < a.N) o[i] = f32_to_bf16_bits(v[i]);
    }
  } else {
    float* o;
    int64_t ld;
    if (EPI == kEpiStoreF32) {
      o = static_cast<float*>(a.out) + static_cast<int64_t>(m) * a.ldo + n0;
      ld = a.ldo;
    } else {
      o = a.partial + (static_cast<int64_t>(split) * a.M + m) * a.N + n0;
      ld = a.N;
    }
    if (n0 + 16 <= a.N && (ld & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        reinterpret_cast<float4*>(o)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (n0 + i < a.N) o[i] = v[i];
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epi_store16(const GemmKernelArgs& a, int m, int n0, int split,
                                            const float (&v)[16]) {
  epi_store16_impl<EPI == kEpiF32Argmax ? kEpiStoreF32 : EPI>(a, m, n0, split, v);
}

// SiLU * mul with PyTorch eager rounding points: g, u are the bf16 GEMM
// outputs; silu(g) = g / (1 + exp(-g)) in fp32 rounded to bf16, product rounded
// to bf16 (respect/system/fused.py:106-113).
__device__ __forceinline__ float silu_mul_bf16(float g_acc, float u_acc) {
  const float g = round_bf16(g_acc);
  const float u = round_bf16(u_acc);
  const float s = round_bf16(g / (1.0f + expf(-g)));
  return __fmul_rn(s, u);
}

// 256 threads: warps 0-3 run the pipeline (weight producer, MMA, TMEM owner,
// token producer); in the epilogue all 8 warps drain TMEM, warp w serving
// lanes 32*(w%4).. and one half of the tile's 16-column chunks.
constexpr int kGemmThreads = 256;

template <int BN, int MT, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                const __grid_constant__ CUtensorMap tmo, const GemmKernelArgs a) {
  using C = GemmCfg<BN, MT, gemm_w_stage_cap(EPI, MT)>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  // barriers: wfull[kWStages], wempty[kWStages], xfull[2], xempty[2], accum
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * C::kWStages + 2 * C::kXStages + 1);
  const uint32_t wfull0 = smem_u32(bars);
  const uint32_t wempty0 = smem_u32(bars + C::kWStages);
  const uint32_t xfull0 = smem_u32(bars + 2 * C::kWStages);
  const uint32_t xempty0 = smem_u32(bars + 2 * C::kWStages + C::kXStages);
  const uint32_t accum = smem_u32(bars + 2 * C::kWStages + 2 * C::kXStages);
  const uint32_t sW = smem_u32(smem + C::kWOff), sX = smem_u32(smem + C::kXOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, split = blockIdx.y, m_group = blockIdx.z;
  const int kc0 = static_cast<int>(static_cast<int64_t>(split) * a.k_chunks / a.splits);
  const int kc1 = static_cast<int>(static_cast<int64_t>(split + 1) * a.k_chunks / a.splits);
  const int nk = kc1 - kc0;
  pdl_trigger();

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tmx);
    tma_prefetch_desc(&tmw);
    if (a.tma_out) tma_prefetch_desc(&tmo);
    for (int s = 0; s < C::kWStages; ++s) {
      mbar_init(wfull0 + 8 * s, 1);
      mbar_init(wempty0 + 8 * s, 1);
    }
    for (int s = 0; s < C::kXStages; ++s) {
      mbar_init(xfull0 + 8 * s, 1);
      mbar_init(xempty0 + 8 * s, 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // Weight producer: contiguous BN x 64 tiles, kWStages deep. Weights never
    // depend on the previous kernel, so this thread does not wait for it (PDL).
    const uint64_t pol_w = policy_evict_first();
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kWStages;
      if (i >= C::kWStages && !mbar_wait(wempty0 + 8 * s, ((i / C::kWStages) & 1) ^ 1, 0x101)) break;
      const int kc = kc0 + i;
      mbar_arrive_expect_tx(wfull0 + 8 * s, C::kWTileBytes);
      tma_load_2d(sW + s * C::kWTileBytes, &tmw, wfull0 + 8 * s, a.w_tiled ? 0 : kc * kBK,
                  a.w_tiled ? (n_tile * a.k_chunks + kc) * BN : n_tile * BN, pol_w);
    }
  } else if (warp == 3 && lane == 0) {
    // Token producer: the activations come from the previous kernel.
    pdl_wait();
    const uint64_t pol_x = policy_evict_last();
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::kXStages;
      if (i >= C::kXStages && !mbar_wait(xempty0 + 8 * s, ((i / C::kXStages) & 1) ^ 1, 0x104)) break;
      mbar_arrive_expect_tx(xfull0 + 8 * s, C::kXStageBytes);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        tma_load_2d(sX + s * C::kXStageBytes + mt * kXTileBytes, &tmx, xfull0 + 8 * s, (kc0 + i) * kBK,
                    (m_group * MT + mt) * kTileM, pol_x);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: 4 K-steps of 16 per stage, one MMA per token tile per step.
    constexpr uint32_t idesc = idesc_bf16_f32(kTileM, BN);
    bool ok = true;
    for (int i = 0; i < nk; ++i) {
      const int sw = i % C::kWStages, sx = i % C::kXStages;
      if (!mbar_wait(wfull0 + 8 * sw, (i / C::kWStages) & 1, 0x102) ||
          !mbar_wait(xfull0 + 8 * sx, (i / C::kXStages) & 1, 0x105)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk) {
        const uint64_t bdesc = sdesc_kmajor_sw128(sW + sw * C::kWTileBytes + kk * 32);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const uint64_t adesc = sdesc_kmajor_sw128(sX + sx * C::kXStageBytes + mt * kXTileBytes + kk * 32);
          umma_bf16(tmem + mt * C::kAccStride, adesc, bdesc, idesc, (i | kk) != 0 ? 1u : 0u);
        }
      }
      // free the stages for the producers (only stages that will be refilled)
      if (i + C::kWStages < nk) umma_commit(wempty0 + 8 * sw);
      if (i + C::kXStages < nk) umma_commit(xempty0 + 8 * sx);
    }
    if (ok) umma_commit(accum);
  }
  __syncwarp();
  pdl_wait();  // outputs are written after the previous kernel has completed

  // Epilogue: warp w owns TMEM lanes [32(w%4), 32(w%4)+32) = token rows of each
  // tile, and chunk half w/4 of the tile's columns.
  // tcgen05.ld is warp-collective: the whole warp takes the same branch.
  // One verdict for the whole CTA (the staged epilogue below has block barriers).
  const bool ok = __syncthreads_and(mbar_wait(accum, 0, 0x103)) != 0;
  tc_fence_after();
  constexpr bool kSilu = EPI == kEpiSiluMul;
  constexpr int kOutCols = kSilu ? BN / 2 : BN;  // output columns of one tile
  constexpr int kRowBytes = gemm_stage_row_bytes(EPI, BN);  // staged box row: 128 or 64 bytes (0: not staged)
  constexpr bool kCanStage = kRowBytes > 0;
  if constexpr (kCanStage) {
    if (ok && a.tma_out) {
      // Staged epilogue: the tile goes to shared memory (the weight ring, idle
      // once the accumulator is final) as boxes of 128 rows x kRowBytes in the
      // matching TMA swizzle (16-byte piece j of row r at j ^ (r & 7) for
      // 128-byte rows, j ^ ((r >> 1) & 3) for 64-byte rows), then one thread
      // writes the boxes with TMA tiled stores: whole lines instead of every
      // thread storing its own row in 16-byte pieces. Rows >= M and columns
      // >= N are clipped by the tensor map.
      constexpr int kElem = gemm_out_elem_bytes(EPI);
      constexpr int kBoxCols = kRowBytes / kElem;
      constexpr int kBoxes = kOutCols / kBoxCols;
      constexpr int kBoxBytes = kTileM * kRowBytes;
      constexpr int kPieces = 16 * kElem / 16;  // 16-byte pieces per 16-column chunk
      static_assert(kBoxes * kBoxBytes <= C::kWStages * C::kWTileBytes, "staging fits in the weight ring");
      uint8_t* stage = smem + C::kWOff;
      const int q4 = warp & 3, hf = warp >> 2;
      const int r = q4 * 32 + lane;
      const int sw = kRowBytes == 128 ? (r & 7) : ((r >> 1) & 3);
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
      uint8_t* srow = stage + r * kRowBytes;
      constexpr int kChunks = kOutCols / 16, kHalfC = (kChunks + 1) / 2;
      const int c_lo = hf * kHalfC, c_hi = min(kChunks, c_lo + kHalfC);
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const int m = (m_group * MT + mt) * kTileM + r;
        unsigned long long best = 0;
        int ex0 = 0, ex1 = 0;
        if (EPI == kEpiF32Argmax) { ex0 = a.excl[0]; ex1 = ex0 + a.excl[1]; }
#pragma unroll 1
        for (int c = c_lo; c < c_hi; ++c) {
          uint32_t w[16 * kElem / 4];
          if constexpr (kSilu) {
            float g[16], u[16];
            tmem_ld16(lane_base + mt * C::kAccStride + c * 16, g);
            tmem_ld16(lane_base + mt * C::kAccStride + BN / 2 + c * 16, u);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              w[i] = pack_bf16x2(silu_mul_bf16(g[2 * i], u[2 * i]), silu_mul_bf16(g[2 * i + 1], u[2 * i + 1]));
          } else {
            float v[16];
            tmem_ld16(lane_base + mt * C::kAccStride + c * 16, v);
            if constexpr (kElem == 2) {
#pragma unroll
              for (int i = 0; i < 8; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(v[i]);
            }
            if constexpr (EPI == kEpiF32Argmax) {
              const int n0 = n_tile * BN + c * 16;
              if (m < a.M) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int n = n0 + i;
                  if (n < a.N && (n < ex0 || n >= ex1)) {
                    const unsigned long long k = argmax_key(v[i], n);
                    best = k > best ? k : best;
                  }
                }
              }
            }
          }
          const int col_bytes = (c * 16 % kBoxCols) * kElem;
          uint8_t* box = srow + (c * 16 / kBoxCols) * kBoxBytes;
#pragma unroll
          for (int i = 0; i < kPieces; ++i)
            *reinterpret_cast<uint4*>(box + (((col_bytes >> 4) + i) ^ sw) * 16) =
                make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
        }
        if (EPI == kEpiF32Argmax && m < a.M && best != 0) atomicMax(a.keys + m, best);
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the TMA engine
        __syncthreads();
        const int row0 = (m_group * MT + mt) * kTileM;
        if (threadIdx.x == 0 && row0 < a.M) {
          const int out_n = kSilu ? a.N / 2 : a.N;  // boxes start inside the tensor; the tail is clipped
#pragma unroll 1
          for (int b = 0; b < kBoxes; ++b) {
            const int x = n_tile * kOutCols + b * kBoxCols;
            if (x >= out_n) break;
            const uint32_t src = smem_u32(stage + b * kBoxBytes);
            if constexpr (EPI == kEpiPartial) tma_store_3d(&tmo, src, x, row0, split);
            else tma_store_2d(&tmo, src, x, row0);
          }
          bulk_commit();
          bulk_wait_read();  // the staging tile has been read
        }
        __syncthreads();  // the staging tile may be refilled / the CTA may exit
      }
    }
  }
  if (ok && !(kCanStage && a.tma_out)) {
    const int q4 = warp & 3, hf = warp >> 2;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
#pragma unroll 1
    for (int mt = 0; mt < MT; ++mt) {
      const int m = (m_group * MT + mt) * kTileM + q4 * 32 + lane;
      if (EPI == kEpiSiluMul) {
        constexpr int kChunks = BN / 32, kHalf = (kChunks + 1) / 2;
        const int c_lo = hf * kHalf, c_hi = min(kChunks, c_lo + kHalf);
#pragma unroll 1
        for (int c = c_lo; c < c_hi; ++c) {
          float g[16], u[16];
          tmem_ld16(lane_base + mt * C::kAccStride + c * 16, g);
          tmem_ld16(lane_base + mt * C::kAccStride + BN / 2 + c * 16, u);
          if (m < a.M) {
#pragma unroll
            for (int i = 0; i < 16; ++i) g[i] = silu_mul_bf16(g[i], u[i]);
            // Output width is N / 2; BN/2 output columns per weight tile.
            GemmKernelArgs b = a;
            b.N = a.N / 2;
            epi_store16<kEpiStoreBF16>(b, m, n_tile * (BN / 2) + c * 16, split, g);
          }
        }
      } else {
        constexpr int kChunks = BN / 16, kHalf = (kChunks + 1) / 2;
        const int c_lo = hf * kHalf, c_hi = min(kChunks, c_lo + kHalf);
        unsigned long long best = 0;
        int ex0 = 0, ex1 = 0;
        if (EPI == kEpiF32Argmax) { ex0 = a.excl[0]; ex1 = ex0 + a.excl[1]; }
#pragma unroll 1
        for (int c = c_lo; c < c_hi; ++c) {
          float v[16];
          tmem_ld16(lane_base + mt * C::kAccStride + c * 16, v);
          const int n0 = n_tile * BN + c * 16;
          if (m < a.M && n0 < a.N) {
            epi_store16<EPI>(a, m, n0, split, v);
            if (EPI == kEpiF32Argmax) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int n = n0 + i;
                if (n < a.N && (n < ex0 || n >= ex1)) {
                  const unsigned long long k = argmax_key(v[i], n);
                  best = k > best ? k : best;
                }
              }
            }
          }
        }
        if (EPI == kEpiF32Argmax && m < a.M && best != 0) atomicMax(a.keys + m, best);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// --------------------------------------------------------------------- host
GemmShape gemm_plan(int M, int N, int K, int num_sms, int force_bn, int force_splits) {
  GemmShape s{};
  s.M = M; s.N = N; s.K = K;
  s.k_chunks = (K + kBK - 1) / kBK;
  int bn = 256;
  if (force_bn) {
    bn = force_bn;
  } else {
    const int n256 = (N + 255) / 256;
    // Few weight tiles over a short K: 128-wide tiles with half the K splits.
    // A split GEMM writes splits x M x N fp32 partials that the next kernel
    // sums, and fewer splits halve that traffic; it pays while each CTA's
    // activation re-reads (K / splits columns per tile) stay short. Measured on
    // the config-3 step: faster for q|k|v (N 4608, K 3584) and o (3584 x 3584),
    // slower for down (K 18944), which keeps 256.
    if (n256 * 4 <= num_sms && s.k_chunks <= 128) bn = 128;
    if (n256 > num_sms) {
      // Many weight tiles: pick the width whose last wave is the fullest.
      const int cands[3] = {256, 208, 128};
      double best = -1.0;
      for (int c : cands) {
        const int t = (N + c - 1) / c;
        const int waves = (t + num_sms - 1) / num_sms;
        const double eff = static_cast<double>(t) / (static_cast<double>(waves) * num_sms);
        if (eff > best + 0.02) { best = eff; bn = c; }
      }
    }
  }
  s.BN = bn;
  s.n_tiles = (N + bn - 1) / bn;
  int splits = 1;
  if (force_splits) {
    splits = force_splits;
  } else if (s.n_tiles < num_sms) {
    splits = std::max(1, std::min(num_sms / s.n_tiles, s.k_chunks / 4));
  }
  s.splits = std::max(1, std::min(splits, s.k_chunks));
  s.mt = M > kTileM ? 2 : 1;
  s.m_groups = (M + kTileM * s.mt - 1) / (kTileM * s.mt);
  return s;
}

int gemm_encode_x(CUtensorMap* m, const void* x, int M, int K, int64_t ldx) {
  return encode_2d_bf16(m, x, K, M, ldx, kBK, kTileM);
}
int gemm_encode_w(CUtensorMap* m, const void* w, int N, int K, int64_t ldw, int BN) {
  return encode_2d_bf16(m, w, K, N, ldw, kBK, BN);
}

size_t gemm_packed_elems(int N, int K, int BN) {
  const size_t nt = (N + BN - 1) / BN, kc = (K + kBK - 1) / kBK;
  return nt * kc * BN * kBK;
}

int gemm_encode_w_packed(CUtensorMap* m, const void* wp, int N, int K, int BN) {
  const uint64_t rows = gemm_packed_elems(N, K, BN) / kBK;
  return encode_2d_bf16(m, wp, kBK, rows, kBK, kBK, BN);
}

// out[((nt*KC + kc)*BN + r)*64 + c] = w[nt*BN + r][kc*64 + c] (zero outside [N, K]).
__global__ void pack_weight_kernel(const uint16_t* __restrict__ w, int64_t ldw, int N, int K, int BN, int KC,
                                   uint16_t* __restrict__ out, int64_t pieces) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= pieces) return;
  const int c8 = static_cast<int>(t % (kBK / 8));
  const int64_t row = t / (kBK / 8);  // packed row = (nt*KC + kc)*BN + r
  const int r = static_cast<int>(row % BN);
  const int64_t tk = row / BN;
  const int kc = static_cast<int>(tk % KC);
  const int nt = static_cast<int>(tk / KC);
  const int n = nt * BN + r, k = kc * kBK + c8 * 8;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (n < N && k < K) v = *reinterpret_cast<const uint4*>(w + static_cast<int64_t>(n) * ldw + k);  // K % 8 == 0
  *reinterpret_cast<uint4*>(out + row * kBK + c8 * 8) = v;
}

int gemm_pack_weight(const void* w, int64_t ldw, int N, int K, int BN, void* out, cudaStream_t st) {
  if (!w || !out || N <= 0 || K <= 0 || K % 8 || ldw % 8 || ldw < K || BN % 16 || BN < 16 || BN > 256)
    return RB_ERR_INVALID_ARG;
  if (!aligned16(w) || !aligned16(out)) return RB_ERR_UNSUPPORTED;
  const int KC = (K + kBK - 1) / kBK;
  const int64_t pieces = static_cast<int64_t>(gemm_packed_elems(N, K, BN) / 8);
  pack_weight_kernel<<<static_cast<unsigned>((pieces + 255) / 256), 256, 0, st>>>(
      static_cast<const uint16_t*>(w), ldw, N, K, BN, KC, static_cast<uint16_t*>(out), pieces);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

template <int BN, int MT, int EPI>
static int launch_t(const GemmShape& s, const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mo,
                    const GemmKernelArgs& ka, cudaStream_t stream, bool pdl) {
  using C = GemmCfg<BN, MT, gemm_w_stage_cap(EPI, MT)>;
  auto kern = gemm_kernel<BN, MT, EPI>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes) != cudaSuccess)
    return RB_ERR_CUDA;
  // all of the unified L1 / shared memory as shared: two capped-ring CTAs per SM
  if (gemm_w_stage_cap(EPI, MT) < 12 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return RB_ERR_CUDA;
  dim3 grid(s.n_tiles, s.splits, s.m_groups);
  return launch_k(kern, grid, dim3(kGemmThreads), C::kSmemBytes, stream, pdl, mx, mw, mo, ka);
}

template <int BN, int MT>
static int launch_epi(const GemmShape& s, const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mo,
                      const GemmKernelArgs& ka, int epi, cudaStream_t stream, bool pdl) {
  switch (epi) {
    case kEpiStoreBF16: return launch_t<BN, MT, kEpiStoreBF16>(s, mx, mw, mo, ka, stream, pdl);
    case kEpiStoreF32: return launch_t<BN, MT, kEpiStoreF32>(s, mx, mw, mo, ka, stream, pdl);
    case kEpiSiluMul: return launch_t<BN, MT, kEpiSiluMul>(s, mx, mw, mo, ka, stream, pdl);
    case kEpiPartial: return launch_t<BN, MT, kEpiPartial>(s, mx, mw, mo, ka, stream, pdl);
    case kEpiF32Argmax: return launch_t<BN, MT, kEpiF32Argmax>(s, mx, mw, mo, ka, stream, pdl);
  }
  return RB_ERR_INVALID_ARG;
}

int gemm_launch_maps(const GemmShape& s, const CUtensorMap& mx, const CUtensorMap& mw,
                     const GemmLaunch& a, cudaStream_t stream, bool pdl) {
  GemmKernelArgs ka{};
  ka.M = s.M; ka.N = s.N; ka.K = s.K;
  ka.k_chunks = s.k_chunks;
  ka.splits = s.splits;
  ka.w_tiled = a.w_tiled;

  ka.out = a.out;
  ka.ldo = a.ldo;
  ka.partial = a.partial;
  ka.keys = a.keys;
  ka.excl = a.excl;
  if (a.epi == kEpiPartial ? a.partial == nullptr : a.out == nullptr) return RB_ERR_INVALID_ARG;
  if (a.epi == kEpiF32Argmax && (!a.keys || !a.excl)) return RB_ERR_INVALID_ARG;
  if (a.epi != kEpiPartial && s.splits != 1) return RB_ERR_INVALID_ARG;
  if (a.epi == kEpiSiluMul && (s.N % s.BN) != 0) return RB_ERR_UNSUPPORTED;
  // Output tensor map for the staged (TMA store) epilogue where the layout allows it.
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  ka.tma_out = 0;
  const int row_bytes = gemm_stage_row_bytes(a.epi, s.BN);
  const int elem = gemm_out_elem_bytes(a.epi);
  const CUtensorMapSwizzle swz = row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType dt = elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const uint32_t box_cols = row_bytes > 0 ? static_cast<uint32_t>(row_bytes / elem) : 0;
  if (row_bytes > 0 && a.epi == kEpiPartial) {
    if (s.N % 4 == 0 && aligned16(a.partial)) {
      const uint64_t dims[3] = {static_cast<uint64_t>(s.N), static_cast<uint64_t>(s.M),
                                static_cast<uint64_t>(s.splits)};
      const uint64_t strides[2] = {static_cast<uint64_t>(s.N) * 4, static_cast<uint64_t>(s.M) * s.N * 4};
      const uint32_t box[3] = {box_cols, kTileM, 1};
      ka.tma_out = encode_tiled(&mo, dt, 3, a.partial, dims, strides, box, swz) == RB_OK;
    }
  } else if (row_bytes > 0) {
    const int out_n = a.epi == kEpiSiluMul ? s.N / 2 : s.N;
    if ((a.ldo * elem) % 16 == 0 && aligned16(a.out)) {
      const uint64_t dims[2] = {static_cast<uint64_t>(out_n), static_cast<uint64_t>(s.M)};
      const uint64_t strides[1] = {static_cast<uint64_t>(a.ldo) * elem};
      const uint32_t box[2] = {box_cols, kTileM};
      ka.tma_out = encode_tiled(&mo, dt, 2, a.out, dims, strides, box, swz) == RB_OK;
    }
  }
  const int key = s.BN * 4 + s.mt;
  switch (key) {
    case 256 * 4 + 1: return launch_epi<256, 1>(s, mx, mw, mo, ka, a.epi, stream, pdl);
    case 256 * 4 + 2: return launch_epi<256, 2>(s, mx, mw, mo, ka, a.epi, stream, pdl);
    case 208 * 4 + 1: return launch_epi<208, 1>(s, mx, mw, mo, ka, a.epi, stream, pdl);
    case 208 * 4 + 2: return launch_epi<208, 2>(s, mx, mw, mo, ka, a.epi, stream, pdl);
    case 128 * 4 + 1: return launch_epi<128, 1>(s, mx, mw, mo, ka, a.epi, stream, pdl);
    case 128 * 4 + 2: return launch_epi<128, 2>(s, mx, mw, mo, ka, a.epi, stream, pdl);
  }
  return RB_ERR_UNSUPPORTED;
}

int gemm_launch(const GemmShape& s, const GemmLaunch& a, cudaStream_t stream) {
  CUtensorMap mx, mw;
  int st = gemm_encode_x(&mx, a.x, s.M, s.K, a.ldx);
  if (st != RB_OK) return st;
  st = gemm_encode_w(&mw, a.w, s.N, s.K, a.ldw, s.BN);
  if (st != RB_OK) return st;
  return gemm_launch_maps(s, mx, mw, a, stream, false);
}

// ------------------------------------------------------------ split-K reduce
template <int OUT_F32>
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N,
                                     void* __restrict__ out, int64_t ldo) {
  const int m = blockIdx.y;
  const int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (n >= N) return;
  const int64_t plane = static_cast<int64_t>(M) * N;
  const float* p = partial + static_cast<int64_t>(m) * N + n;
  if (n + 4 <= N && (N & 3) == 0) {
    float4 acc = *reinterpret_cast<const float4*>(p);
    for (int s = 1; s < splits; ++s) {
      const float4 t = *reinterpret_cast<const float4*>(p + s * plane);
      acc.x += t.x; acc.y += t.y; acc.z += t.z; acc.w += t.w;
    }
    if (OUT_F32) {
      float* o = static_cast<float*>(out) + static_cast<int64_t>(m) * ldo + n;
      o[0] = acc.x; o[1] = acc.y; o[2] = acc.z; o[3] = acc.w;
    } else {
      uint16_t* o = static_cast<uint16_t*>(out) + static_cast<int64_t>(m) * ldo + n;
      o[0] = f32_to_bf16_bits(acc.x); o[1] = f32_to_bf16_bits(acc.y);
      o[2] = f32_to_bf16_bits(acc.z); o[3] = f32_to_bf16_bits(acc.w);
    }
  } else {
    for (int j = n; j < n + 4 && j < N; ++j) {
      float acc = p[j - n];
      for (int s = 1; s < splits; ++s) acc += p[j - n + s * plane];
      if (OUT_F32) static_cast<float*>(out)[static_cast<int64_t>(m) * ldo + j] = acc;
      else static_cast<uint16_t*>(out)[static_cast<int64_t>(m) * ldo + j] = f32_to_bf16_bits(acc);
    }
  }
}

int splitk_reduce(const float* partial, int splits, int M, int N, void* out, int64_t ldo,
                  int out_f32, cudaStream_t stream) {
  if (M <= 0 || N <= 0) return RB_OK;
  dim3 block(256);
  dim3 grid((N + 4 * 256 - 1) / (4 * 256), M);
  if (out_f32) splitk_reduce_kernel<1><<<grid, block, 0, stream>>>(partial, splits, M, N, out, ldo);
  else splitk_reduce_kernel<0><<<grid, block, 0, stream>>>(partial, splits, M, N, out, ldo);
  return cudaGetLastError() == cudaSuccess ? RB_OK : RB_ERR_CUDA;
}

}  // namespace rb
