// Prefix phase of the trie attention on the 5th-generation tensor cores
// (bf16 inputs, head_dim 128). One CTA = one query head x 128 query rows x one
// fixed prefix chunk of prefix_chunk(NP, H) keys at absolute positions; keys are
// processed in tiles of 128 in ascending order (respect/kernels/attention.py:36-50):
//
//   S = Q K^T            tcgen05.mma, M=128 rows, N=128 keys, K=128 dims -> TMEM
//   m' = max(m, rowmax(S*scale)); alpha = 2^(m - m'); p = 2^(S*scale - m')
//   O = O*alpha (in TMEM, by the softmax threads); l = l*alpha + sum(p)
//   O += bf16(p) V       tcgen05.mma, A = P (TMEM, written by the softmax threads), B = V (MN-major)
// The output accumulator never leaves TMEM until the chunk is done, so the
// softmax of tile j+1 runs while the tensor core computes P_j V_j.
//
// Warp roles: warps 0-7 softmax / correction (two threads per query row: warp
// w serves TMEM lanes 32*(w%4).., key / dim columns [64*(w/4), 64*(w/4)+64);
// the row max and row sum of the halves are combined through shared memory,
// lower half first), warp 8 TMA producer (Q once, K/V double-buffered), warp 9
// MMA issuer and TMEM owner. Each row's result depends only on that row and the chunk's keys:
// the MMA computes rows independently and every row reduction runs in a
// fixed order, so a row gives the same bits whatever the other rows are.
#include "attention.cuh"
#include "common.cuh"
#include "host_util.h"

namespace rb {

namespace tc {
constexpr int kRows = 128, kKeys = 128, kD = 128;
constexpr int kHalf = 128 * 64 * 2;          // one 64-element-wide swizzled half tile: 16 KB
constexpr int kQOff = 0;                     // Q: 2 halves
constexpr int kKVOff = 2 * kHalf;            // 2 stages x (K 2 halves, V 2 halves)
constexpr int kStage = 4 * kHalf;            // 64 KB
constexpr int kBarOff = kKVOff + 2 * kStage;   // 160 KB
// TMEM columns: S double buffer 0-255, O 256-383, P (bf16 pairs, 64 columns) from 384
constexpr uint32_t kPCol = 384;
constexpr int kRedOff = kBarOff + 256;       // row max / row sum exchange: [2 tiles][2][2 halves][128] floats
constexpr int kSmem = 1024 + kRedOff + 1024 * 4;
static_assert(kSmem <= 232448, "shared memory budget");
static_assert(kRows * kPartStride * 4 <= 2 * kStage, "partial block staged in the K/V buffers");
constexpr int kSoftmaxThreads = 256;
constexpr int kThreads = kSoftmaxThreads + 64;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
// barrier indices. K and V of a stage have their own full / empty barriers: K is
// free again once Q K^T is done (early in a tile), V once P V is (at its end),
// so the next tile but one's K is requested a whole softmax earlier than a
// shared K/V barrier would allow, which keeps the TMA latency off the critical path.
enum { Q_FULL = 0, K_FULL = 1, V_FULL = 3, K_EMPTY = 5, V_EMPTY = 7, S_FULL = 9, P_FULL = 11, O_FULL = 12, NBAR = 13 };
constexpr float kRescaleSlack = 8.0f;
constexpr uint32_t kIdescQK = idesc_bf16_f32(128, 128, 0, 0);
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 128, 0, 1);
}  // namespace tc

// At most 136 registers: the CTA's 10 warps then leave a register-file partition
// room for two warps of the node kernel (48 registers), which folds beside it.
__global__ void __maxnreg__(136)
    attn_prefix_tc(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const AttnDev p, float* __restrict__ part) {
  using namespace tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBAR);
  auto bar = [&](int i) { return smem_u32(bars + i); };

  const int c = blockIdx.x, h = blockIdx.y, rt = blockIdx.z;
  const int NP = p.sp ? p.sp->prompt_len : p.NP;
  const int M = p.sp ? min(p.M, p.sp->q) : p.M;
  const int C = prefix_chunk(NP, p.H);
  const int k0 = c * C;
  const int k1 = min(NP, k0 + C);
  // Dependents (the node kernel) are released only after this grid's wait: they
  // read q and the node K / V before their own wait, so every CTA, including
  // one without work, releases them only once the kernel before this one is done.
  if (k0 >= k1 || rt * kRows >= M) {  // uniform per CTA, before any barrier exists
    pdl_wait();
    return;
  }
  const int ntiles = (k1 - k0 + kKeys - 1) / kKeys;
  const int kvh = h / (p.H / p.HK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
    mbar_init(bar(Q_FULL), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(K_FULL + i), 1);
      mbar_init(bar(V_FULL + i), 1);
      mbar_init(bar(K_EMPTY + i), 1);
      mbar_init(bar(V_EMPTY + i), 1);
    }
    mbar_init(bar(S_FULL), 1);
    mbar_init(bar(S_FULL + 1), 1);
    mbar_init(bar(P_FULL), kSoftmaxThreads);
    mbar_init(bar(O_FULL), 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q / K / V come from the previous kernels
  pdl_trigger();
  const uint32_t sQ = smem_u32(smem + kQOff), sKV = smem_u32(smem + kKVOff);

  if (warp == kProducerWarp) {
    if (lane == 0) {  // TMA producer
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(bar(Q_FULL), 2 * kHalf);
      tma_load_3d(sQ, &tq, bar(Q_FULL), 0, rt * kRows, h, pol);
      tma_load_3d(sQ + kHalf, &tq, bar(Q_FULL), 64, rt * kRows, h, pol);
      // K(j) and V(j) in the order their stages free up (K(j) after Q K^T of
      // tile j-2, V(j) after P V of tile j-2).
      for (int j = 0; j < ntiles; ++j) {
        const int s = j & 1;
        const uint32_t st = sKV + s * kStage;
        const int key = k0 + j * kKeys;
        if (j >= 2 && !mbar_wait(bar(K_EMPTY + s), ((j >> 1) & 1) ^ 1, 0x211)) break;
        mbar_arrive_expect_tx(bar(K_FULL + s), 2 * kHalf);
        tma_load_3d(st, &tk, bar(K_FULL + s), 0, key, kvh, pol);
        tma_load_3d(st + kHalf, &tk, bar(K_FULL + s), 64, key, kvh, pol);
        if (j >= 2 && !mbar_wait(bar(V_EMPTY + s), ((j >> 1) & 1) ^ 1, 0x21a)) break;
        mbar_arrive_expect_tx(bar(V_FULL + s), 2 * kHalf);
        tma_load_3d(st + 2 * kHalf, &tv, bar(V_FULL + s), 0, key, kvh, pol);
        tma_load_3d(st + 3 * kHalf, &tv, bar(V_FULL + s), 64, key, kvh, pol);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {  // MMA issuer
      auto issue_qk = [&](int j) {
        const uint32_t st = sKV + (j & 1) * kStage;
        const uint32_t d = tmem + (j & 1) * 128;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
          umma_bf16(d, sdesc_kmajor_sw128(sQ + off), sdesc_kmajor_sw128(st + off), kIdescQK, kk ? 1u : 0u);
        }
        umma_commit(bar(S_FULL + (j & 1)));
        if (j + 2 < ntiles) umma_commit(bar(K_EMPTY + (j & 1)));  // K(j) read: the stage takes K(j+2)
      };
      bool ok = mbar_wait(bar(Q_FULL), 0, 0x212) && mbar_wait(bar(K_FULL), 0, 0x213);
      if (ok) {
        tc_fence_after();
        issue_qk(0);
      }
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles) {
          if (!mbar_wait(bar(K_FULL + ((j + 1) & 1)), ((j + 1) >> 1) & 1, 0x214)) break;
          tc_fence_after();
          issue_qk(j + 1);
        }
        // P_j written and O rescaled by alpha_j (both signalled by P_FULL), V_j loaded
        if (!mbar_wait(bar(P_FULL), j & 1, 0x215) || !mbar_wait(bar(V_FULL + (j & 1)), (j >> 1) & 1, 0x21b))
          break;
        tc_fence_after();
        const uint32_t sv = sKV + (j & 1) * kStage + 2 * kHalf;
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          // A = P from tensor memory: keys 16kk .. 16kk + 15 are columns kPCol + 8kk ..
          umma_bf16_ta(tmem + 256, tmem + kPCol + kk * 8, sdesc_mnmajor_sw128(sv + kk * 2048, kHalf), kIdescPV,
                       (j | kk) ? 1u : 0u);
        }
        umma_commit(bar(O_FULL));
        if (j + 2 < ntiles) umma_commit(bar(V_EMPTY + (j & 1)));  // V(j) read: the stage takes V(j+2)
      }
    }
  } else {
    // Softmax / correction. Thread (warp w, lane): row r = 32*(w%4) + lane,
    // columns [64*hf, 64*hf + 64) of S (keys) and of O (dims), hf = w / 4.
    const int q4 = warp & 3, hf = warp >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    // Row max / row sum exchange, double-buffered by tile parity: tile j's
    // sums are read after tile j+1's max barrier (every thread has written
    // them by then), so a tile needs one block barrier, not two.
    float* red_all = reinterpret_cast<float*>(smem + kRedOff);  // [2 (tile)][2 (max|sum)][2 (half)][128] floats
    const float scale2 = p.sm_scale * 1.4426950408889634f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    // A timed-out wait (device error already raised) skips this warp's TMEM
    // work but never a named barrier, so the other warps cannot block.
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(S_FULL + (j & 1)), (j >> 1) & 1, 0x217));
      const uint32_t sb = lane_base + (j & 1) * 128 + hf * 64;
      const int nvalid = min(kKeys, k1 - (k0 + j * kKeys)) - hf * 64;  // valid keys in this half (may be <= 0)
      uint32_t raw[4][16];
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) tmem_ld16_nowait(sb + cc * 16, raw[cc]);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int i = 0; i < 16; ++i) raw[cc][i] = 0u;
      }
      // Row max on the raw scores (scale2 > 0 and rounding are monotone, so
      // max(s)*scale2 == max(s*scale2)); keys past the chunk end are masked.
      if (nvalid < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= nvalid) raw[i >> 4][i & 15] = __float_as_uint(-INFINITY);
      }
      // pairwise tree (max is exact, so any grouping gives the same value)
      float t32[32];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        t32[i] = fmaxf(__uint_as_float(raw[i >> 4][i & 15]), __uint_as_float(raw[(i + 32) >> 4][(i + 32) & 15]));
#pragma unroll
      for (int w2 = 16; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int i = 0; i < w2; ++i) t32[i] = fmaxf(t32[i], t32[i + w2]);
      float mx = t32[0];
      float* red = red_all + (j & 1) * 512;
      red[hf * 128 + r] = mx * scale2;
      named_bar(1, kSoftmaxThreads);
      mx = fmaxf(red[r], red[128 + r]);
      if (j > 0) {  // the previous tile's row sum, now written by both halves
        const float* prev = red_all + ((j - 1) & 1) * 512 + 256;
        l = fmaf(l, alpha_prev, prev[r] + prev[128 + r]);
      }
      // Lazy rescaling: the running max moves (and O, l are rescaled) only when
      // the tile's max exceeds it by more than kRescaleSlack (log2 units);
      // otherwise the stale max stays and p = 2^(s - m) may reach 2^kRescaleSlack,
      // well inside bf16 and fp32 range. O / l is unchanged mathematically, the
      // O round trip through TMEM is skipped in most tiles, and the decision
      // depends on the row's own scores only.
      const float m_new = (mx > m + kRescaleSlack) ? mx : m;  // finite after the first tile (valid keys)
      const float alpha = fast_exp2(m - m_new);
      const float neg_m = -m_new;
      uint32_t w[32];
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        // p = 2^(s*scale2 - m'); a masked key (-inf) gives exactly 0
        const float p0 = fast_exp2(fmaf(__uint_as_float(raw[i >> 4][i & 15]), scale2, neg_m));
        const float p1 = fast_exp2(fmaf(__uint_as_float(raw[(i + 1) >> 4][(i + 1) & 15]), scale2, neg_m));
        t32[i / 2] = p0 + p1;  // the row sum: a fixed pairwise tree over the 64 keys
        w[i / 2] = pack_bf16x2(p0, p1);
      }
#pragma unroll
      for (int w2 = 16; w2 >= 1; w2 >>= 1)
#pragma unroll
        for (int i = 0; i < w2; ++i) t32[i] += t32[i + w2];
      const float rs = t32[0];
      red[256 + hf * 128 + r] = rs;
      if (j > 0 && ok) {
        // P_{j-1} V_{j-1} must be complete before P_j overwrites P and O is rescaled.
        ok = __all_sync(0xffffffffu, mbar_wait(bar(O_FULL), (j - 1) & 1, 0x218));
        // alpha == 1 for every row of the warp: O * 1 == O, skip the round trip
        if (ok && !__all_sync(0xffffffffu, alpha == 1.0f)) {
          tc_fence_after();
          const uint32_t ob = lane_base + 256 + hf * 64;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) tmem_ld16_nowait(ob + cc * 16, raw[cc]);
          tmem_wait_ld();
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
            for (int i = 0; i < 16; ++i) raw[cc][i] = __float_as_uint(__uint_as_float(raw[cc][i]) * alpha);
            tmem_st16(ob + cc * 16, raw[cc]);
          }
          tmem_wait_st();
        }
      }
      if (ok) {  // P of this thread's row and 64 keys: columns kPCol + 32 hf .. + 31 of its lane
        const uint32_t pb = lane_base + kPCol + hf * 32;
        uint32_t w0[16], w1[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) { w0[i] = w[i]; w1[i] = w[16 + i]; }
        tmem_st16(pb, w0);
        tmem_st16(pb + 16, w1);
        tmem_wait_st();
      }
      tc_fence_before();         // S loads, O and P stores of this tile ordered before the arrive
      mbar_arrive(bar(P_FULL));
      alpha_prev = alpha;
      m = m_new;
    }
    named_bar(1, kSoftmaxThreads);  // the last tile's row sums
    if (ntiles > 0) {
      const float* prev = red_all + ((ntiles - 1) & 1) * 512 + 256;
      l = fmaf(l, alpha_prev, prev[r] + prev[128 + r]);
    }
    // the last P V product, then O leaves TMEM once
    float acc[64];
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(O_FULL), (ntiles - 1) & 1, 0x219));
    if (ok) {
      tc_fence_after();
      uint32_t raw[4][16];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld16_nowait(lane_base + 256 + hf * 64 + cc * 16, raw[cc]);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 64; ++i) acc[i] = __uint_as_float(raw[i >> 4][i & 15]);
    }
    // The 128 rows' partials are one contiguous block of the partial buffer
    // ([row][kPartStride] floats): stage it in the K/V buffers (free once the
    // last P V is done) and write it with one bulk copy.
    const int row = rt * kRows + r;
    float* st = reinterpret_cast<float*>(smem + kKVOff) + r * kPartStride;
    if (ok && row < M) {
#pragma unroll
      for (int i = 0; i < 64; i += 4)
        *reinterpret_cast<float4*>(st + hf * 64 + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
      if (hf == 0) *reinterpret_cast<float4*>(st + kD) = make_float4(m, l, 0.f, 0.f);
    }
    fence_proxy_async_smem();
    named_bar(1, kSoftmaxThreads);
    if (threadIdx.x == 0) {
      const int rows = min(kRows, M - rt * kRows);
      bulk_store(part + ((static_cast<int64_t>(c) * p.H + h) * p.M + rt * kRows) * kPartStride, sKV,
                 static_cast<uint32_t>(rows * kPartStride * 4));
      bulk_commit();
      bulk_wait_read();  // the staging block has been read before the CTA may exit
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// [H, rows, 128] bf16 (rows `ld_row` elements apart, heads `ld_head` apart) as a
// 3-D tensor map with 64 x 128 x 1 boxes.
int encode_heads_3d(CUtensorMap* m, const void* base, int rows, int heads, int64_t ld_row, int64_t ld_head) {
  const uint64_t dims[3] = {128, static_cast<uint64_t>(rows), static_cast<uint64_t>(heads)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld_row) * 2, static_cast<uint64_t>(ld_head) * 2};
  const uint32_t box[3] = {64, 128, 1};
  return encode_tiled(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int attn_prefix_tc_launch(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttnDev& p,
                          float* part, int nchunks, cudaStream_t stream, bool pdl) {
  if (cudaFuncSetAttribute(attn_prefix_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::kSmem) != cudaSuccess)
    return RB_ERR_CUDA;
  dim3 grid(nchunks, p.H, (p.M + tc::kRows - 1) / tc::kRows);
  return launch_k(attn_prefix_tc, grid, dim3(tc::kThreads), tc::kSmem, stream, pdl, tq, tk, tv, p, part);
}

}  // namespace rb
