// Deterministic trie-verification attention (respect/kernels/attention.py:15-96).
//
// Phase 1 (prefix, keys [0, NP)): the prefix is cut into chunks of
// C = prefix_chunk(NP, H) keys at ABSOLUTE positions (chunk c = [c*C, (c+1)*C)), each
// chunk reduced by an online softmax over fixed key tiles into a partial
// (max, sum, acc[D]) per query row. Chunk boundaries depend on NP only.
// Phase 2 (per query row and kv head, one warp): fold the row's ALLOWED node
// keys in their list order (committed slots, then trie ancestors; or slot order
// in the mask modes), in batches cut at fixed list positions, into a node
// partial; then merge the chunk partials in chunk order and the node partial.
// Masked slots are skipped, which is exactly what the reference's -inf scores
// do (exp(-inf) = 0, alpha = 1), so a row's result depends only on the values of
// its allowed keys and their order, never on where siblings sit in the buffer
// or on how many rows the call carries. Final acc / l, one cast. Both phases run
// on the tensor cores: bf16 products (tcgen05 / mma.sync), or for fp32 data three
// tf32 products per term.
#include "attention.cuh"
#include "common.cuh"
#include "host_util.h"

namespace rb {

constexpr float kLog2e = 1.4426950408889634f;

template <typename T> __device__ __forceinline__ float ldf(const T* p);
template <> __device__ __forceinline__ float ldf<float>(const float* p) { return *p; }
template <> __device__ __forceinline__ float ldf<uint16_t>(const uint16_t* p) { return bf16_bits_to_f32(*p); }

// Loads 4 consecutive elements as fp32.
template <typename T> __device__ __forceinline__ void ld4(const T* p, float (&v)[4]);
template <> __device__ __forceinline__ void ld4<float>(const float* p, float (&v)[4]) {
  const float4 t = *reinterpret_cast<const float4*>(p);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
template <> __device__ __forceinline__ void ld4<uint16_t>(const uint16_t* p, float (&v)[4]) {
  const uint2 t = *reinterpret_cast<const uint2*>(p);
  v[0] = bf16_bits_to_f32(static_cast<uint16_t>(t.x));
  v[1] = bf16_bits_to_f32(static_cast<uint16_t>(t.x >> 16));
  v[2] = bf16_bits_to_f32(static_cast<uint16_t>(t.y));
  v[3] = bf16_bits_to_f32(static_cast<uint16_t>(t.y >> 16));
}

// ----------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  // src_bytes = 0 copies nothing and zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// ----------------------------------------------------------------- prefix (fp32 data, tensor cores)
// fp32 data on the tensor cores. Each score and each P·V term is the sum of
// three tf32 products, hi·hi + hi·lo + lo·hi (q: hi = tf32(x) rounded to
// nearest, ties away, lo = tf32(x - hi); K, V and P: hi = x truncated to tf32,
// lo = x - hi): at most about 2^-19 relative error per term, fp32 accumulation
// (mma.sync.m16n8k8 tf32, independent of the row count).
//
// Block = 4 warps = 16 query rows of one head over one prefix chunk. Warp w
// takes keys 8w .. 8w + 7 of every 32-key tile (one n-tile of S, one k-step of
// P·V), copies their K and V rows into its own shared-memory rows with cp.async
// (software-pipelined: S of the next keys runs before P·V of the current ones)
// and keeps its own online-softmax state, so the warps never wait for
// one another until the end, where the four states are merged in warp order
// into the chunk partial.
//
// Fragment layouts (lane = 4g + t): the 128 head dims enter the S products in a
// fixed permuted order, k-step 2i + o (o = 0, 1) position t <- dim 16i + 4t + 2o
// and position t + 4 <- dim 16i + 4t + 2o + 1, so that a lane's A (q) and B (k)
// values of two k-steps are one float4. The P·V k-step takes the warp's 8 keys in
// the order (0, 2, 4, 6 | 1, 3, 5, 7), which makes S's accumulator fragment the P
// A-fragment as it stands; P·V n-tile j, position n <- dim 32(j / 4) + 4n + j % 4,
// so a lane's V values of four n-tiles are one float4.
namespace t32 {
// Warps per block, each a key group of 8 within a tile (5 and 6 measured slower:
// 57.6 and 52.2 us against 45.3 for config 1, fewer blocks fit on an SM).
constexpr int kWarps = 4;
constexpr int kRows = 16, kTK = 8 * kWarps, kD = 128;
constexpr int kQP = 144, kKP = 144, kVP = 132;   // shared-memory row pitches (floats): conflict-free fragment reads
constexpr int kQFloats = kRows * kQP;            // one of Q hi / Q lo
constexpr int kWarpKV = 8 * kKP + 8 * kVP;               // one warp's K and V rows
constexpr int kMergeFloats = kWarps * kRows * kPartStride;   // the warps' states (reuses the K / V rows)
static_assert(kMergeFloats <= kWarps * kWarpKV, "merge area fits in the K / V rows");
constexpr int kSmemBytes = (2 * kQFloats + kWarps * kWarpKV) * 4;
}  // namespace t32

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// d (16x8 fp32) += a (16x8 tf32, row-major) * b (8x8 tf32, column-major)
__device__ __forceinline__ void mma_tf32_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// d += (ah + al)(bh + bl) without the al·bl term
__device__ __forceinline__ void mma_3xtf32(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                           uint32_t bh0, uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma_tf32_1688(d, ah[0], ah[1], ah[2], ah[3], bh0, bh1);
  mma_tf32_1688(d, ah[0], ah[1], ah[2], ah[3], bl0, bl1);
  mma_tf32_1688(d, al[0], al[1], al[2], al[3], bh0, bh1);
}
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - __uint_as_float(hi));
}
// The per-tile split of K, V and P on the integer and FMA pipes (the conversion
// above runs on the slower multi-function pipe): hi = x with the 13 low mantissa
// bits cleared, lo = x - hi (exact), whose own low bits the tf32 MMA drops:
// |x - hi - lo_tf32| < 2^-20 |x|.
__device__ __forceinline__ void split_tf32_fast(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xFFFFE000u;
  lo = __float_as_uint(x - __uint_as_float(hi));
}

__global__ void __launch_bounds__(32 * t32::kWarps) attn_prefix_tf32(const AttnDev p, float* __restrict__ part) {
  using namespace t32;
  extern __shared__ __align__(16) float t32_smem[];
  uint32_t* qh = reinterpret_cast<uint32_t*>(t32_smem);          // [16][kQP] tf32 hi of q
  uint32_t* ql = qh + kQFloats;                                  // [16][kQP] tf32 lo of q
  float* kv0 = t32_smem + 2 * kQFloats;                          // per warp: K [8][kKP], V [8][kVP]
  const int c = blockIdx.x, h = blockIdx.y, r0 = blockIdx.z * kRows;
  const int kvh = h / (p.H / p.HK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  float* ks = kv0 + warp * kWarpKV;   // this warp's K rows
  float* vs = ks + 8 * kKP;           // and V rows
  // Dependents (the node kernel) are released only after this grid's wait: they
  // read q and the node K / V before their own wait.
  pdl_wait();
  pdl_trigger();
  const int NP = p.sp ? p.sp->prompt_len : p.NP;
  const int M = p.sp ? min(p.M, p.sp->q) : p.M;
  const int C = prefix_chunk(NP, p.H);
  const int k0 = c * C;
  const int k1 = min(NP, k0 + C);
  if (k0 >= k1 || r0 >= M) return;  // chunk beyond the prefix / rows beyond the live ones
  const float* q = static_cast<const float*>(p.q);
  const float* kp = static_cast<const float*>(p.kp);
  const float* vp = static_cast<const float*>(p.vp);
  for (int i = threadIdx.x; i < kRows * kD; i += blockDim.x) {
    const int r = i / kD, d = i % kD;
    const float x = (r0 + r < M) ? q[h * p.sqh + static_cast<int64_t>(r0 + r) * p.sqm + d] : 0.f;
    uint32_t hi, lo;
    split_tf32(x, hi, lo);
    qh[r * kQP + d] = hi;
    ql[r * kQP + d] = lo;
  }
  const float scale2 = p.sm_scale * kLog2e;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // rows g and g + 8
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  __syncthreads();   // q visible to every warp
  // K or V rows of the warp's keys kw .. kw + 7 (keys past the chunk end zero-filled), one cp.async group
  auto load8 = [&](float* dst, int pitch, const float* src, int64_t sh, int64_t sn, int kw) {
    const float* base = src + kvh * sh + 4 * lane;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const bool ok = kw + r < k1;
      cp_async16(dst + r * pitch + 4 * lane, base + static_cast<int64_t>(ok ? kw + r : k0) * sn, ok ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // S of the warp's keys kw .. kw + 7 into s (16 rows x 8 keys)
  auto s_products = [&](float (&s)[4]) {
    // S (16 rows x the warp's 8 keys). Six independent accumulators (hi·hi,
    // hi·lo, lo·hi, each for even and odd k-steps) keep the MMA chains short;
    // they are added in a fixed order at the end.
    float acc[6][4];
#pragma unroll
    for (int a = 0; a < 6; ++a)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][e] = 0.f;
    const float* kr = ks + g * kKP + 4 * t;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 a_g = *reinterpret_cast<const uint4*>(qh + g * kQP + 16 * i + 4 * t);
      const uint4 a_g8 = *reinterpret_cast<const uint4*>(qh + (g + 8) * kQP + 16 * i + 4 * t);
      const uint4 b_g = *reinterpret_cast<const uint4*>(ql + g * kQP + 16 * i + 4 * t);
      const uint4 b_g8 = *reinterpret_cast<const uint4*>(ql + (g + 8) * kQP + 16 * i + 4 * t);
      const float4 kv = *reinterpret_cast<const float4*>(kr + 16 * i);
      uint32_t kh[4], kl[4];
      split_tf32_fast(kv.x, kh[0], kl[0]);
      split_tf32_fast(kv.y, kh[1], kl[1]);
      split_tf32_fast(kv.z, kh[2], kl[2]);
      split_tf32_fast(kv.w, kh[3], kl[3]);
      // k-step 2i: dims 16i + 4t + {0, 1}; k-step 2i + 1: dims 16i + 4t + {2, 3}
      mma_tf32_1688(acc[0], a_g.x, a_g8.x, a_g.y, a_g8.y, kh[0], kh[1]);
      mma_tf32_1688(acc[1], a_g.z, a_g8.z, a_g.w, a_g8.w, kh[2], kh[3]);
      mma_tf32_1688(acc[2], a_g.x, a_g8.x, a_g.y, a_g8.y, kl[0], kl[1]);
      mma_tf32_1688(acc[3], a_g.z, a_g8.z, a_g.w, a_g8.w, kl[2], kl[3]);
      mma_tf32_1688(acc[4], b_g.x, b_g8.x, b_g.y, b_g8.y, kh[0], kh[1]);
      mma_tf32_1688(acc[5], b_g.z, b_g8.z, b_g.w, b_g8.w, kh[2], kh[3]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) s[e] = (acc[0][e] + acc[1][e]) + ((acc[2][e] + acc[3][e]) + (acc[4][e] + acc[5][e]));
  };
  // online softmax of those keys; P (tf32 hi / lo) into ph / pl
  uint32_t ph[4], pl[4];
  auto softmax_step = [&](int kw, float (&s)[4]) {
    // online softmax over the 8 keys (rows g: s[0], s[1]; rows g + 8: s[2], s[3])
    const bool v0 = kw + 2 * t < k1, v1 = kw + 2 * t + 1 < k1;
    s[0] = v0 ? s[0] * scale2 : -INFINITY;
    s[1] = v1 ? s[1] * scale2 : -INFINITY;
    s[2] = v0 ? s[2] * scale2 : -INFINITY;
    s[3] = v1 ? s[3] * scale2 : -INFINITY;
    float x0 = fmaxf(s[0], s[1]), x1 = fmaxf(s[2], s[3]);
    x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, 1));
    x0 = fmaxf(x0, __shfl_xor_sync(0xffffffffu, x0, 2));
    x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, 1));
    x1 = fmaxf(x1, __shfl_xor_sync(0xffffffffu, x1, 2));
    const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);   // finite: the warp's first key is valid
    const float al0 = fast_exp2(m0 - n0), al1 = fast_exp2(m1 - n1);
    const float p0 = fast_exp2(s[0] - n0), p1 = fast_exp2(s[1] - n0);
    const float p2 = fast_exp2(s[2] - n1), p3 = fast_exp2(s[3] - n1);
    float rs0 = p0 + p1, rs1 = p2 + p3;
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
    l0 = fmaf(l0, al0, rs0);
    l1 = fmaf(l1, al1, rs1);
    m0 = n0;
    m1 = n1;
    if (!__all_sync(0xffffffffu, al0 == 1.f && al1 == 1.f)) {   // the warp's running maxima moved
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= al0; o[j][1] *= al0;
        o[j][2] *= al1; o[j][3] *= al1;
      }
    }
    // A of P V = P in key order (2t, 2t + 1) -> positions (t, t + 4)
    split_tf32_fast(p0, ph[0], pl[0]);   // (g, key 2t)
    split_tf32_fast(p2, ph[1], pl[1]);   // (g + 8, key 2t)
    split_tf32_fast(p1, ph[2], pl[2]);   // (g, key 2t + 1)
    split_tf32_fast(p3, ph[3], pl[3]);   // (g + 8, key 2t + 1)
  };
  // O += P V of the keys whose V rows are staged
  auto pv_step = [&]() {
    const float* v0r = vs + (2 * t) * kVP + 4 * g;
    const float* v1r = v0r + kVP;
#pragma unroll
    for (int jq = 0; jq < 4; ++jq) {
      const float4 va = *reinterpret_cast<const float4*>(v0r + 32 * jq);
      const float4 vb = *reinterpret_cast<const float4*>(v1r + 32 * jq);
      const float a4[4] = {va.x, va.y, va.z, va.w}, b4[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int jr = 0; jr < 4; ++jr) {
        uint32_t h0, l0b, h1, l1b;
        split_tf32_fast(a4[jr], h0, l0b);
        split_tf32_fast(b4[jr], h1, l1b);
        mma_3xtf32(o[jq * 4 + jr], ph, pl, h0, h1, l0b, l1b);
      }
    }
  };
  // Software-pipelined over the warp's tiles: S of the next keys runs before
  // P·V of the current ones, so each V load lands during a softmax and the
  // next S products, each K load during a P·V and a softmax.
  // cp.async groups in flight at each wait: K(next), V(current).
  const int kfirst = k0 + warp * 8;
  if (kfirst < k1) {
    load8(ks, kKP, kp, p.skph, p.skpn, kfirst);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    float s[4];
    s_products(s);
    __syncwarp();   // every lane is done with these K rows
    if (kfirst + kTK < k1) load8(ks, kKP, kp, p.skph, p.skpn, kfirst + kTK);
    else asm volatile("cp.async.commit_group;" ::: "memory");   // an empty group keeps the counts
    load8(vs, kVP, vp, p.svph, p.svpn, kfirst);
    softmax_step(kfirst, s);
  }
  for (int kw = kfirst; kw < k1; kw += kTK) {
    const int kn = kw + kTK;   // the warp's keys in the next tile
    float s[4];
    if (kn < k1) {
      asm volatile("cp.async.wait_group 1;" ::: "memory");   // K(next) (V(current) may pend)
      __syncwarp();
      s_products(s);
      __syncwarp();
      if (kn + kTK < k1) load8(ks, kKP, kp, p.skph, p.skpn, kn + kTK);
      else asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
    asm volatile("cp.async.wait_group 1;" ::: "memory");     // V(current)
    __syncwarp();
    pv_step();
    __syncwarp();   // every lane is done with these V rows
    if (kn < k1) {
      load8(vs, kVP, vp, p.svph, p.svpn, kn);
      softmax_step(kn, s);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();   // every warp is done with its K / V rows: the merge area reuses them
  // merge the warps' states in warp order: O = sum_w O_w 2^(m_w - m), l likewise
  float* st = kv0;   // [4][16][kPartStride]: O at dims 0..127, m at 128, l at 129
  float* mine = st + warp * kRows * kPartStride;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 32 * (j >> 2) + 8 * t + (j & 3);
    mine[g * kPartStride + d] = o[j][0];
    mine[g * kPartStride + d + 4] = o[j][1];
    mine[(g + 8) * kPartStride + d] = o[j][2];
    mine[(g + 8) * kPartStride + d + 4] = o[j][3];
  }
  if (t == 0) {
    mine[g * kPartStride + 128] = m0;
    mine[g * kPartStride + 129] = l0;
    mine[(g + 8) * kPartStride + 128] = m1;
    mine[(g + 8) * kPartStride + 129] = l1;
  }
  __syncthreads();
  // thread (row r, dims 16 q .. 16 q + 15)
  const int r = threadIdx.x >> 3, d0 = (threadIdx.x & 7) * 16;
  if (r >= kRows) return;
  if (r0 + r >= M) return;
  float mw[kWarps], mx = -INFINITY;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    mw[w] = st[(w * kRows + r) * kPartStride + 128];
    mx = fmaxf(mx, mw[w]);
  }
  float acc[16], lsum = 0.f;
#pragma unroll
  for (int e = 0; e < 16; ++e) acc[e] = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    if (mw[w] == -INFINITY) continue;   // a warp without keys in this chunk
    const float a = fast_exp2(mw[w] - mx);
    const float* src = st + (w * kRows + r) * kPartStride;
    lsum = fmaf(src[129], a, lsum);
#pragma unroll
    for (int e = 0; e < 16; ++e) acc[e] = fmaf(src[d0 + e], a, acc[e]);
  }
  float* dst = part + ((static_cast<int64_t>(c) * p.H + h) * p.M + r0 + r) * kPartStride;
#pragma unroll
  for (int e = 0; e < 16; e += 4)
    *reinterpret_cast<float4*>(dst + d0 + e) = make_float4(acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
  if (d0 == 0) {
    dst[128] = mx;
    dst[129] = lsum;
  }
}

// ----------------------------------------------------------------- node phase
__device__ __forceinline__ bool node_allowed(const AttnDev& p, int row, int j) {
  switch (p.mask_kind) {
    case RB_MASK_BOOL:
      return static_cast<const uint8_t*>(p.msk)[row * p.smm + j * p.smn] != 0;
    case RB_MASK_ADD_BF16:
      return (static_cast<const uint16_t*>(p.msk)[row * p.smm + j * p.smn] & 0x7FFFu) == 0;
    case RB_MASK_ADD_F32:
      return static_cast<const float*>(p.msk)[row * p.smm + j * p.smn] == 0.f;
    default:
      return j <= row + p.causal_first;
  }
}

// Node phase. One item = one query row x one kv head (the G = H / HK query
// heads of the kv head together). A row's key list (committed slots, then its
// trie ancestors; or the slots its mask allows, in slot order) is folded in
// batches cut at fixed list positions, so a row's node partial depends only on
// its keys and their order; the output is merge(prefix chunk 0, 1, ..., node
// partial), in that order. The folds need only q and the node K / V, so they run
// before griddepcontrol.wait (under PDL, beside the prefix kernel); the merges
// with the prefix chunk partials after it.
constexpr int kMaxGroup = 16;   // query heads per kv head: one m16 tile of rows

// Running softmax state of one (row, head), lane-owned dims [4*lane, 4*lane+4).
struct NodeAcc {
  float m, l, acc[4];
};

// Fold `b` into `a` as the later piece: a = merge(a, b). Empty pieces (m = -inf) are skipped.
__device__ __forceinline__ void merge_into(NodeAcc& a, float bm, float bl, const float (&bacc)[4]) {
  if (bm == -INFINITY) return;
  const float m_new = fmaxf(a.m, bm);
  const float x = fast_exp2(a.m - m_new);
  const float y = fast_exp2(bm - m_new);
#pragma unroll
  for (int e = 0; e < 4; ++e) a.acc[e] = fmaf(bacc[e], y, a.acc[e] * x);
  a.l = fmaf(bl, y, a.l * x);
  a.m = m_new;
}

// ----------------------------------------------------------------- node phase, bf16 (tensor cores)
// One warp per item (query row x kv head) folds the row's ordered key list (the
// committed slots, then its trie ancestors root first; in the mask modes, the
// allowed slots in slot order) for all G query heads of the kv head at once, in
// batches of 32 list entries counted from the start of the list:
//   S = Q K_list^T          mma.sync m16n8k16 (heads padded to 16 rows), fp32
//   m' = max(m, rowmax(S*scale)); a = 2^(m - m'); P = 2^(S*scale - m')
//   O = O*a + bf16(P) V_list   mma.sync, fp32 accumulators; l = l*a + rowsum(P)
// The MMAs group keys by their position in that list, never by their slot in
// the KV buffer, and a trie node's list is the same sequence as the token-by-token
// step's (its committed keys), so a committed row gets the same bits either way.
// Row maxima and sums combine the four threads of a quad by shuffles in a fixed
// order. After griddepcontrol.wait the node partial is merged with the prefix
// chunk partials (chunk order, node partial last), as in attn_nodes.
namespace nm {
constexpr int kPitch = 136;                       // bf16 elements per staged row (272 bytes: ldmatrix conflict-free)
constexpr int kQRows = 16, kListRows = 32;
constexpr int kQBytes = kQRows * kPitch * 2;      // 4352
constexpr int kKVBytes = kListRows * kPitch * 2;  // 8704 each for K and V
constexpr int kStageBytes = kQBytes + 2 * kKVBytes;
// staging | node partials [G][kPartStride] | list slots [kListRows] | mbarrier of the merge's bulk copies
__host__ __device__ inline int smem_bytes(int G) { return kStageBytes + G * kPartStride * 4 + kListRows * 4 + 16; }
}  // namespace nm

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
// d (16x8 fp32) += a (16x16 bf16, row-major) * b (16x8 bf16, column-major)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(32) attn_nodes_mma(const AttnDev p, const float* __restrict__ part) {
  using namespace nm;
  extern __shared__ __align__(16) uint8_t nsm[];
  uint16_t* Qs = reinterpret_cast<uint16_t*>(nsm);
  uint16_t* Ks = reinterpret_cast<uint16_t*>(nsm + kQBytes);
  uint16_t* Vs = reinterpret_cast<uint16_t*>(nsm + kQBytes + kKVBytes);
  const int G = p.H / p.HK;
  float* npart = reinterpret_cast<float*>(nsm + kStageBytes);                   // [G][kPartStride]
  int* slots = reinterpret_cast<int*>(nsm + kStageBytes + G * kPartStride * 4);  // [kListRows]
  const int lane = threadIdx.x, g = lane >> 2, c = lane & 3;
  const int live = p.sp ? p.sp->q : p.M;
  const int row = blockIdx.x % p.M, kvh = blockIdx.x / p.M;
  const uint32_t sbar = smem_u32(nsm + kStageBytes + G * kPartStride * 4 + kListRows * 4);
  pdl_trigger();
  if (lane == 0) {
    mbar_init(sbar, 1);
    fence_mbar_init();
  }
  for (int h = lane; h < G; h += 32) npart[h * kPartStride + 128] = -INFINITY;   // empty node partial

  if (row < live) {
    // ---- the node fold (needs only q and the node K / V: runs before the wait)
    const int NP = p.sp ? p.sp->prompt_len : p.NP;
    const uint16_t* kn = p.kn ? static_cast<const uint16_t*>(p.kn)
                              : static_cast<const uint16_t*>(p.kp) + static_cast<int64_t>(NP) * p.skpn;
    const uint16_t* vn = p.vn ? static_cast<const uint16_t*>(p.vn)
                              : static_cast<const uint16_t*>(p.vp) + static_cast<int64_t>(NP) * p.svpn;
    const int64_t kbase = static_cast<int64_t>(kvh) * p.sknh, vbase = static_cast<int64_t>(kvh) * p.svnh;
    const bool trie = p.mask_kind == kMaskTrie;
    int base = 0, depth = -1;
    const int32_t* chain = nullptr;
    if (trie) {
      base = p.sp ? p.sp->base : p.causal_first;
      depth = p.depths[row];
      if (depth < 0 || depth > row || depth >= p.chain_ld) depth = -1;  // invalid trie: reported when the chain was built
      chain = p.chain + static_cast<int64_t>(row) * p.chain_ld;
    }
    // q rows of the group's heads (8-byte pieces; rows past G are zero)
    const uint16_t* q = static_cast<const uint16_t*>(p.q);
    for (int i = lane; i < kQRows * 32; i += 32) {
      const int r = i >> 5, pc = i & 31;
      uint2 v = make_uint2(0u, 0u);
      if (r < G) v = *reinterpret_cast<const uint2*>(q + (kvh * G + r) * p.sqh + static_cast<int64_t>(row) * p.sqm + pc * 4);
      *reinterpret_cast<uint2*>(Qs + r * kPitch + pc * 4) = v;
    }
    float o[16][4];
#pragma unroll
    for (int d = 0; d < 16; ++d)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[d][e] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // query heads g and g + 8
    const float scale2 = p.sm_scale * kLog2e;
    const int total = trie ? base + depth + 1 : p.NN;
    const uint32_t sQ = smem_u32(Qs), sK = smem_u32(Ks), sV = smem_u32(Vs);
    // Batches are cut at fixed positions of the row's key list (every 32 list
    // entries from its start), whatever slots the entries occupy: the candidates
    // (list positions in trie mode, slots in the mask modes) are scanned in order
    // and the allowed ones appended to slots[] until 32 are held or none remain.
    int scan = 0;   // next candidate to examine
    while (scan < total) {
      // 1. the next (up to) 32 list entries
      int cnt = 0;
      __syncwarp();   // the previous batch's reads of slots / K / V are done (and q is staged)
      while (cnt < kListRows && scan < total) {
        const int i = scan + lane;
        int slot = 0;
        bool v;
        if (trie) {
          const int ci = i - base;
          const int cv = (ci >= 0 && ci < p.chain_ld) ? chain[ci] : 0;
          v = i < total;
          slot = i < base ? i : base + cv;
        } else {
          v = i < total && node_allowed(p, row, i);
          slot = i;
        }
        const unsigned bits = __ballot_sync(0xffffffffu, v);
        const int rank = __popc(bits & ((1u << lane) - 1u)), room = kListRows - cnt;
        if (v && rank < room) slots[cnt + rank] = slot;
        const int n = __popc(bits);
        if (n <= room) {
          cnt += n;
          scan += 32;
        } else {   // the window holds more than fits: resume at its first entry left out
          const unsigned left = __ballot_sync(0xffffffffu, v && rank == room);
          scan += __ffs(left) - 1;
          cnt = kListRows;
        }
      }
      __syncwarp();
      if (cnt == 0) break;
      // 2. stage the entries' K and V rows (rows past cnt zero-filled)
      for (int it = 0; it < kListRows / 2; ++it) {
        const int u = it * 2 + (lane >> 4), pc = lane & 15;
        const bool ok = u < cnt;
        const int64_t sl = ok ? slots[u] : 0;
        cp_async16(Ks + u * kPitch + pc * 8, kn + kbase + sl * p.sknn + pc * 8, ok ? 16u : 0u);
        cp_async16(Vs + u * kPitch + pc * 8, vn + vbase + sl * p.svnn + pc * 8, ok ? 16u : 0u);
      }
      asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      // 3. S = Q K^T over the 32 entries (four 8-entry tiles)
      float sc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[j][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        const int qr = (lane & 7) + ((lane >> 3) & 1) * 8, qc = kk * 16 + (lane >> 4) * 8;
        ldsm_x4(sQ + (qr * kPitch + qc) * 2, a0, a1, a2, a3);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t b0r, b1r;
          const int kr = j * 8 + (lane & 7), kc = kk * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x2(sK + (kr * kPitch + kc) * 2, b0r, b1r);
          mma_bf16_16816(sc[j], a0, a1, a2, a3, b0r, b1r);
        }
      }
      // 4. online softmax of rows g and g + 8 (entries past cnt masked)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (j * 8 + 2 * c + e >= cnt) sc[j][e] = sc[j][2 + e] = -INFINITY;
          mx0 = fmaxf(mx0, sc[j][e]);
          mx1 = fmaxf(mx1, sc[j][2 + e]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n0 = fmaxf(m0, mx0 * scale2), n1 = fmaxf(m1, mx1 * scale2);
      const float al0 = fast_exp2(m0 - n0), al1 = fast_exp2(m1 - n1);
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sc[j][e] = fast_exp2(fmaf(sc[j][e], scale2, -n0));
          sc[j][2 + e] = fast_exp2(fmaf(sc[j][2 + e], scale2, -n1));
          rs0 += sc[j][e];
          rs1 += sc[j][2 + e];
        }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = fmaf(l0, al0, rs0);
      l1 = fmaf(l1, al1, rs1);
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int d = 0; d < 16; ++d) {
        o[d][0] *= al0; o[d][1] *= al0;
        o[d][2] *= al1; o[d][3] *= al1;
      }
      // 5. O += P V over the 32 entries (two 16-entry k-steps). The node keys'
      // weights stay fp32 in the reference (attention.py:59-66, p * v in fp32),
      // so P goes in as two bf16 parts, hi = bf16(p) and lo = bf16(p - hi)
      // (p to about 16 significant bits), each times the bf16 V rows.
      uint32_t pa[2][4], pl[2][4];
#pragma unroll
      for (int kc = 0; kc < 2; ++kc)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int j = 2 * kc + (i >> 1), e = (i & 1) * 2;   // pieces: (j, e), (j, e + 1)
          const float h0 = round_bf16(sc[j][e]), h1 = round_bf16(sc[j][e + 1]);
          pa[kc][i] = pack_bf16x2(h0, h1);
          pl[kc][i] = pack_bf16x2(sc[j][e] - h0, sc[j][e + 1] - h1);
        }
#pragma unroll
      for (int d = 0; d < 16; ++d)
#pragma unroll
        for (int kc = 0; kc < 2; ++kc) {
          uint32_t b0r, b1r;
          ldsm_x2_t(sV + ((kc * 16 + (lane & 15)) * kPitch + d * 8) * 2, b0r, b1r);
          mma_bf16_16816(o[d], pa[kc][0], pa[kc][1], pa[kc][2], pa[kc][3], b0r, b1r);
          mma_bf16_16816(o[d], pl[kc][0], pl[kc][1], pl[kc][2], pl[kc][3], b0r, b1r);
        }
    }
    // the node partial of every head of the group: acc[128], m, l
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int h = g + half * 8;
      if (h < G) {
        float* np = npart + h * kPartStride;
#pragma unroll
        for (int d = 0; d < 16; ++d) {
          np[d * 8 + 2 * c] = o[d][2 * half];
          np[d * 8 + 2 * c + 1] = o[d][2 * half + 1];
        }
        if (c == 0) {
          np[128] = half ? m1 : m0;
          np[129] = half ? l1 : l0;
        }
      }
    }
  }

  pdl_wait();  // the prefix chunk partials are complete
  const int NP = p.sp ? p.sp->prompt_len : p.NP;
  const int nchunks = prefix_nchunks(NP, p.H);
  const int d0 = lane * 4;
  uint16_t* out = static_cast<uint16_t*>(p.out) + static_cast<int64_t>(row) * p.som + d0;
  if (row >= live) {  // padding row of a bucketed engine step: zeros, no reads
    for (int h = 0; h < G; ++h)
      *reinterpret_cast<uint2*>(out + (kvh * G + h) * p.soh) = make_uint2(0u, 0u);
    return;
  }
  // The row's chunk partials (every head of the group) are copied into the
  // staging area with all copies in flight; all of them when they fit (config 3:
  // 5 chunks x 7 heads), else one head's chunks at a time.
  constexpr int kPiece = kPartStride * 4;
  float* pieces = reinterpret_cast<float*>(nsm);
  const int cap_pieces = kStageBytes / kPiece;
  const bool all_at_once = G * nchunks <= cap_pieces;
  // One bulk copy per piece (the TMA engine moves each 528-byte piece), all
  // completing on one mbarrier: a single round trip instead of a lane-by-lane
  // stream of 16-byte copies.
  uint32_t sphase = 0;
  auto stage = [&](int h_first, int h_count) {   // pieces (chunk k, head h_first + j) at index j * nchunks + k
    fence_proxy_async_smem();   // this lane's generic reads of the staging area come before the copies' writes
    __syncwarp();
    const int n = h_count * nchunks;
    if (lane == 0) mbar_arrive_expect_tx(sbar, static_cast<uint32_t>(n * kPiece));
    __syncwarp();
    for (int pi = lane; pi < n; pi += 32) {
      const int k = pi % nchunks, hh = h_first + pi / nchunks;
      const float* src = part + ((static_cast<int64_t>(k) * p.H + kvh * G + hh) * p.M + row) * kPartStride;
      bulk_load(smem_u32(reinterpret_cast<uint8_t*>(pieces) + pi * kPiece), src, kPiece, sbar);
    }
    const bool ok = mbar_wait(sbar, sphase, 0x231);
    sphase ^= 1u;
    __syncwarp();
    return ok;
  };
  __syncwarp();   // the node partial written by the fold is visible to every lane
  if (all_at_once && nchunks > 0 && !stage(0, G)) return;
  for (int h = 0; h < G; ++h) {
    if (!all_at_once && nchunks > 0 && !stage(h, 1)) return;
    const float* ph = pieces + (all_at_once ? h * nchunks : 0) * kPartStride;
    // prefix chunk partials in ascending chunk order, then the node partial
    NodeAcc r{-INFINITY, 0.f, {0.f, 0.f, 0.f, 0.f}};
    for (int k = 0; k < nchunks; ++k) {
      const float* o = ph + k * kPartStride;
      const float4 v = *reinterpret_cast<const float4*>(o + d0);
      const float ca[4] = {v.x, v.y, v.z, v.w};
      merge_into(r, o[128], o[129], ca);
    }
    const float* np = npart + h * kPartStride;
    const float4 v = *reinterpret_cast<const float4*>(np + d0);
    const float ca[4] = {v.x, v.y, v.z, v.w};
    merge_into(r, np[128], np[129], ca);
    // bf16 output: one correctly rounded reciprocal per head, then products (the
    // reference divides with Triton's fp32 `/`, itself not correctly rounded)
    const float rl = __frcp_rn(r.l);
    uint16_t b[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) b[e] = f32_to_bf16_bits(r.acc[e] * rl);
    *reinterpret_cast<uint2*>(out + (kvh * G + h) * p.soh) =
        make_uint2(static_cast<uint32_t>(b[0]) | (static_cast<uint32_t>(b[1]) << 16),
                   static_cast<uint32_t>(b[2]) | (static_cast<uint32_t>(b[3]) << 16));
  }
}
// ----------------------------------------------------------------- node phase, fp32 (tensor cores)
// The node phase of attn_nodes_mma for fp32 data: the same items (one warp per
// query row x kv head), the same ordered key list cut into batches of 32 by list
// position, the same online softmax and merge, with every q·k and p·v term the
// sum of three tf32 products (hi·hi + hi·lo + lo·hi) as in attn_prefix_tf32.
// S of a batch is four m16n8k8 n-tiles (8 keys each); P·V takes each n-tile as
// one k-step in the key order (0, 2, 4, 6 | 1, 3, 5, 7), so S's accumulator
// fragment is the A fragment. The head dims use the permutations of
// attn_prefix_tf32 (q·k: k-step pair i reads dims 16i + 4t .. +3; P·V n-tile j,
// position n <- dim 32(j / 4) + 4n + j % 4).
namespace nf {
constexpr int kQP = 144, kKP = 144, kVP = 132;   // row pitches (floats): conflict-free fragment reads
constexpr int kQRows = 16, kListRows = 32;
constexpr int kQBytes = 2 * kQRows * kQP * 4;    // tf32 hi and lo of q
constexpr int kKBytes = kListRows * kKP * 4, kVBytes = kListRows * kVP * 4;
constexpr int kStageBytes = kQBytes + kKBytes + kVBytes;
// staging | node partials [G][kPartStride] | list slots | mbarrier of the merge's bulk copies
__host__ __device__ inline int smem_bytes(int G) { return kStageBytes + G * kPartStride * 4 + kListRows * 4 + 16; }
}  // namespace nf

__global__ void __launch_bounds__(32) attn_nodes_tf32(const AttnDev p, const float* __restrict__ part) {
  using namespace nf;
  extern __shared__ __align__(16) uint8_t nsm[];
  uint32_t* Qh = reinterpret_cast<uint32_t*>(nsm);
  uint32_t* Ql = Qh + kQRows * kQP;
  float* Ks = reinterpret_cast<float*>(nsm + kQBytes);
  float* Vs = reinterpret_cast<float*>(nsm + kQBytes + kKBytes);
  const int G = p.H / p.HK;
  float* npart = reinterpret_cast<float*>(nsm + kStageBytes);                   // [G][kPartStride]
  int* slots = reinterpret_cast<int*>(nsm + kStageBytes + G * kPartStride * 4);  // [kListRows]
  const int lane = threadIdx.x, g = lane >> 2, t = lane & 3;
  const int live = p.sp ? p.sp->q : p.M;
  const int row = blockIdx.x % p.M, kvh = blockIdx.x / p.M;
  const uint32_t sbar = smem_u32(nsm + kStageBytes + G * kPartStride * 4 + kListRows * 4);
  pdl_trigger();
  if (lane == 0) {
    mbar_init(sbar, 1);
    fence_mbar_init();
  }
  for (int h = lane; h < G; h += 32) npart[h * kPartStride + 128] = -INFINITY;   // empty node partial

  if (row < live) {
    // ---- the node fold (needs only q and the node K / V: runs before the wait)
    const int NP = p.sp ? p.sp->prompt_len : p.NP;
    const float* kn = p.kn ? static_cast<const float*>(p.kn)
                           : static_cast<const float*>(p.kp) + static_cast<int64_t>(NP) * p.skpn;
    const float* vn = p.vn ? static_cast<const float*>(p.vn)
                           : static_cast<const float*>(p.vp) + static_cast<int64_t>(NP) * p.svpn;
    const int64_t kbase = static_cast<int64_t>(kvh) * p.sknh, vbase = static_cast<int64_t>(kvh) * p.svnh;
    const bool trie = p.mask_kind == kMaskTrie;
    int base = 0, depth = -1;
    const int32_t* chain = nullptr;
    if (trie) {
      base = p.sp ? p.sp->base : p.causal_first;
      depth = p.depths[row];
      if (depth < 0 || depth > row || depth >= p.chain_ld) depth = -1;  // invalid trie: reported when the chain was built
      chain = p.chain + static_cast<int64_t>(row) * p.chain_ld;
    }
    // q rows of the group's heads as tf32 hi / lo (rows past G are zero)
    const float* q = static_cast<const float*>(p.q);
    for (int i = lane; i < kQRows * 128; i += 32) {
      const int r = i >> 7, d = i & 127;
      const float x = r < G ? q[(kvh * G + r) * p.sqh + static_cast<int64_t>(row) * p.sqm + d] : 0.f;
      uint32_t hi, lo;
      split_tf32(x, hi, lo);
      Qh[r * kQP + d] = hi;
      Ql[r * kQP + d] = lo;
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;   // query heads g and g + 8
    const float scale2 = p.sm_scale * kLog2e;
    const int total = trie ? base + depth + 1 : p.NN;
    // Batches are cut at fixed positions of the row's key list, as in attn_nodes_mma.
    int scan = 0;   // next candidate to examine
    while (scan < total) {
      // 1. the next (up to) 32 list entries
      int cnt = 0;
      __syncwarp();   // the previous batch's reads of slots / K / V are done (and q is staged)
      while (cnt < kListRows && scan < total) {
        const int i = scan + lane;
        int slot = 0;
        bool v;
        if (trie) {
          const int ci = i - base;
          const int cv = (ci >= 0 && ci < p.chain_ld) ? chain[ci] : 0;
          v = i < total;
          slot = i < base ? i : base + cv;
        } else {
          v = i < total && node_allowed(p, row, i);
          slot = i;
        }
        const unsigned bits = __ballot_sync(0xffffffffu, v);
        const int rank = __popc(bits & ((1u << lane) - 1u)), room = kListRows - cnt;
        if (v && rank < room) slots[cnt + rank] = slot;
        const int n = __popc(bits);
        if (n <= room) {
          cnt += n;
          scan += 32;
        } else {   // the window holds more than fits: resume at its first entry left out
          const unsigned left = __ballot_sync(0xffffffffu, v && rank == room);
          scan += __ffs(left) - 1;
          cnt = kListRows;
        }
      }
      __syncwarp();
      if (cnt == 0) break;
      // 2. stage the entries' K and V rows (rows past cnt zero-filled); lane = 16 bytes of a row
      for (int u = 0; u < kListRows; ++u) {
        const bool ok = u < cnt;
        const int64_t sl = ok ? slots[u] : 0;
        cp_async16(Ks + u * kKP + 4 * lane, kn + kbase + sl * p.sknn + 4 * lane, ok ? 16u : 0u);
        cp_async16(Vs + u * kVP + 4 * lane, vn + vbase + sl * p.svnn + 4 * lane, ok ? 16u : 0u);
      }
      asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
      __syncwarp();
      // 3. S = Q K^T over the 32 entries (four 8-entry n-tiles)
      float sc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[j][e] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 a_g = *reinterpret_cast<const uint4*>(Qh + g * kQP + 16 * i + 4 * t);
        const uint4 a_g8 = *reinterpret_cast<const uint4*>(Qh + (g + 8) * kQP + 16 * i + 4 * t);
        const uint4 b_g = *reinterpret_cast<const uint4*>(Ql + g * kQP + 16 * i + 4 * t);
        const uint4 b_g8 = *reinterpret_cast<const uint4*>(Ql + (g + 8) * kQP + 16 * i + 4 * t);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 kv = *reinterpret_cast<const float4*>(Ks + (j * 8 + g) * kKP + 16 * i + 4 * t);
          uint32_t kh[4], kl[4];
          split_tf32_fast(kv.x, kh[0], kl[0]);
          split_tf32_fast(kv.y, kh[1], kl[1]);
          split_tf32_fast(kv.z, kh[2], kl[2]);
          split_tf32_fast(kv.w, kh[3], kl[3]);
          // k-step 2i: dims 16i + 4t + {0, 1}; k-step 2i + 1: dims 16i + 4t + {2, 3}
          mma_tf32_1688(sc[j], a_g.x, a_g8.x, a_g.y, a_g8.y, kh[0], kh[1]);
          mma_tf32_1688(sc[j], a_g.z, a_g8.z, a_g.w, a_g8.w, kh[2], kh[3]);
          mma_tf32_1688(sc[j], a_g.x, a_g8.x, a_g.y, a_g8.y, kl[0], kl[1]);
          mma_tf32_1688(sc[j], a_g.z, a_g8.z, a_g.w, a_g8.w, kl[2], kl[3]);
          mma_tf32_1688(sc[j], b_g.x, b_g8.x, b_g.y, b_g8.y, kh[0], kh[1]);
          mma_tf32_1688(sc[j], b_g.z, b_g8.z, b_g.w, b_g8.w, kh[2], kh[3]);
        }
      }
      // 4. online softmax of rows g and g + 8 (entries past cnt masked)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          if (j * 8 + 2 * t + e >= cnt) sc[j][e] = sc[j][2 + e] = -INFINITY;
          mx0 = fmaxf(mx0, sc[j][e]);
          mx1 = fmaxf(mx1, sc[j][2 + e]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n0 = fmaxf(m0, mx0 * scale2), n1 = fmaxf(m1, mx1 * scale2);
      const float al0 = fast_exp2(m0 - n0), al1 = fast_exp2(m1 - n1);
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          sc[j][e] = fast_exp2(fmaf(sc[j][e], scale2, -n0));
          sc[j][2 + e] = fast_exp2(fmaf(sc[j][2 + e], scale2, -n1));
          rs0 += sc[j][e];
          rs1 += sc[j][2 + e];
        }
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
      rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
      rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
      l0 = fmaf(l0, al0, rs0);
      l1 = fmaf(l1, al1, rs1);
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= al0; o[j][1] *= al0;
        o[j][2] *= al1; o[j][3] *= al1;
      }
      // 5. O += P V: n-tile kc of S is the k-step over keys 8kc + (2t, 2t + 1)
#pragma unroll
      for (int kc = 0; kc < 4; ++kc) {
        uint32_t ph[4], pl[4];
        split_tf32_fast(sc[kc][0], ph[0], pl[0]);   // (g, key 2t)
        split_tf32_fast(sc[kc][2], ph[1], pl[1]);   // (g + 8, key 2t)
        split_tf32_fast(sc[kc][1], ph[2], pl[2]);   // (g, key 2t + 1)
        split_tf32_fast(sc[kc][3], ph[3], pl[3]);   // (g + 8, key 2t + 1)
        const float* v0r = Vs + (kc * 8 + 2 * t) * kVP + 4 * g;
        const float* v1r = v0r + kVP;
#pragma unroll
        for (int jq = 0; jq < 4; ++jq) {
          const float4 va = *reinterpret_cast<const float4*>(v0r + 32 * jq);
          const float4 vb = *reinterpret_cast<const float4*>(v1r + 32 * jq);
          const float a4[4] = {va.x, va.y, va.z, va.w}, b4[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
          for (int jr = 0; jr < 4; ++jr) {
            uint32_t h0, l0b, h1, l1b;
            split_tf32_fast(a4[jr], h0, l0b);
            split_tf32_fast(b4[jr], h1, l1b);
            mma_3xtf32(o[jq * 4 + jr], ph, pl, h0, h1, l0b, l1b);
          }
        }
      }
    }
    // the node partial of every head of the group: acc[128], m, l
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int h = g + half * 8;
      if (h < G) {
        float* np = npart + h * kPartStride;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int d = 32 * (j >> 2) + 8 * t + (j & 3);
          np[d] = o[j][2 * half];
          np[d + 4] = o[j][2 * half + 1];
        }
        if (t == 0) {
          np[128] = half ? m1 : m0;
          np[129] = half ? l1 : l0;
        }
      }
    }
  }

  pdl_wait();  // the prefix chunk partials are complete
  const int NP = p.sp ? p.sp->prompt_len : p.NP;
  const int nchunks = prefix_nchunks(NP, p.H);
  const int d0 = lane * 4;
  float* out = static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.som + d0;
  if (row >= live) {  // padding row: zeros, no reads
    for (int h = 0; h < G; ++h)
      *reinterpret_cast<float4*>(out + (kvh * G + h) * p.soh) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  // The row's chunk partials, one bulk copy per 528-byte piece on one mbarrier:
  // all of them when they fit, else one head's chunks at a time.
  constexpr int kPiece = kPartStride * 4;
  float* pieces = reinterpret_cast<float*>(nsm);
  const int cap_pieces = kStageBytes / kPiece;
  const bool all_at_once = G * nchunks <= cap_pieces;
  uint32_t sphase = 0;
  auto stage = [&](int h_first, int h_count) {   // pieces (chunk k, head h_first + j) at index j * nchunks + k
    fence_proxy_async_smem();   // this lane's generic accesses of the staging area come before the copies' writes
    __syncwarp();
    const int n = h_count * nchunks;
    if (lane == 0) mbar_arrive_expect_tx(sbar, static_cast<uint32_t>(n * kPiece));
    __syncwarp();
    for (int pi = lane; pi < n; pi += 32) {
      const int k = pi % nchunks, hh = h_first + pi / nchunks;
      const float* src = part + ((static_cast<int64_t>(k) * p.H + kvh * G + hh) * p.M + row) * kPartStride;
      bulk_load(smem_u32(reinterpret_cast<uint8_t*>(pieces) + pi * kPiece), src, kPiece, sbar);
    }
    const bool ok = mbar_wait(sbar, sphase, 0x232);
    sphase ^= 1u;
    __syncwarp();
    return ok;
  };
  __syncwarp();   // the node partial written by the fold is visible to every lane
  if (all_at_once && nchunks > 0 && !stage(0, G)) return;
  for (int h = 0; h < G; ++h) {
    if (!all_at_once && nchunks > 0 && !stage(h, 1)) return;
    const float* ph = pieces + (all_at_once ? h * nchunks : 0) * kPartStride;
    // prefix chunk partials in ascending chunk order, then the node partial
    NodeAcc r{-INFINITY, 0.f, {0.f, 0.f, 0.f, 0.f}};
    for (int k = 0; k < nchunks; ++k) {
      const float* o = ph + k * kPartStride;
      const float4 v = *reinterpret_cast<const float4*>(o + d0);
      const float ca[4] = {v.x, v.y, v.z, v.w};
      merge_into(r, o[128], o[129], ca);
    }
    const float* np = npart + h * kPartStride;
    const float4 v = *reinterpret_cast<const float4*>(np + d0);
    const float ca[4] = {v.x, v.y, v.z, v.w};
    merge_into(r, np[128], np[129], ca);
    *reinterpret_cast<float4*>(out + (kvh * G + h) * p.soh) =
        make_float4(__fdiv_rn(r.acc[0], r.l), __fdiv_rn(r.acc[1], r.l), __fdiv_rn(r.acc[2], r.l),
                    __fdiv_rn(r.acc[3], r.l));
  }
}

template <typename T>
static int launch_nodes(const AttnDev& p, const float* part, cudaStream_t stream, bool pdl) {
  const int G = p.H / p.HK;
  if (G > kMaxGroup) return RB_ERR_UNSUPPORTED;
  const int items = p.M * p.HK;
  if (items <= 0) return RB_OK;
  if (sizeof(T) == 2) {   // bf16: one warp per item on the tensor cores
    const int dyn = nm::smem_bytes(G);
    if (cudaFuncSetAttribute(attn_nodes_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess)
      return RB_ERR_CUDA;
    return launch_k(attn_nodes_mma, dim3(items), dim3(32), dyn, stream, pdl, p, part);
  }
  static_assert(sizeof(T) == 2 || sizeof(T) == 4, "bf16 or fp32 data");
  // fp32: one warp per item, three tf32 products per term
  const int dyn = nf::smem_bytes(G);
  if (cudaFuncSetAttribute(attn_nodes_tf32, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn) != cudaSuccess)
    return RB_ERR_CUDA;
  return launch_k(attn_nodes_tf32, dim3(items), dim3(32), dyn, stream, pdl, p, part);
}

// ----------------------------------------------------------------- host
size_t attn_workspace_bytes(int H, int M, int D, int NP) {
  (void)D;
  const int nchunks = prefix_nchunks(NP, H);
  return static_cast<size_t>(nchunks > 0 ? nchunks : 1) * H * (M > 0 ? M : 1) * kPartStride * sizeof(float);
}

int attn_validate(const rb_attn_args* a) {
  if (!a) return RB_ERR_INVALID_ARG;
  if (a->dtype != RB_F32 && a->dtype != RB_BF16) return RB_ERR_UNSUPPORTED;
  if (a->H <= 0 || a->HK <= 0 || a->M < 0 || a->NP < 0 || a->NN < 0) return RB_ERR_INVALID_ARG;
  if (a->H % a->HK != 0) return RB_ERR_INVALID_ARG;
  if (a->H / a->HK > kMaxGroup) return RB_ERR_UNSUPPORTED;
  if (a->D != 128) return RB_ERR_UNSUPPORTED;
  if (a->sqd != 1 || a->sod != 1 || (a->NP > 0 && (a->skpd != 1 || a->svpd != 1)) ||
      (a->NN > 0 && (a->sknd != 1 || a->svnd != 1)))
    return RB_ERR_UNSUPPORTED;
  if (!a->q || !a->out || (a->NP > 0 && (!a->kp || !a->vp)) || (a->NN > 0 && (!a->kn || !a->vn)))
    return RB_ERR_INVALID_ARG;
  if (a->mask_kind < RB_MASK_BOOL || a->mask_kind > RB_MASK_CAUSAL) return RB_ERR_INVALID_ARG;
  if (a->mask_kind != RB_MASK_CAUSAL && a->NN > 0 && !a->msk) return RB_ERR_INVALID_ARG;
  // Vector loads of 4 elements need 4-element-aligned row strides and bases
  // (only for the tensors a call actually reads).
  const bool pre = a->NP > 0, nod = a->NN > 0;
  const int64_t strides[] = {a->sqh, a->sqm, a->soh, a->som,
                             pre ? a->skph : 0, pre ? a->skpn : 0, pre ? a->svph : 0, pre ? a->svpn : 0,
                             nod ? a->sknh : 0, nod ? a->sknn : 0, nod ? a->svnh : 0, nod ? a->svnn : 0};
  for (int64_t s : strides)
    if (s % 4 != 0) return RB_ERR_UNSUPPORTED;
  const int eb = a->dtype == RB_F32 ? 4 : 2;
  const void* ptrs[] = {a->q, pre ? a->kp : nullptr, pre ? a->vp : nullptr, nod ? a->kn : nullptr,
                        nod ? a->vn : nullptr, a->out};
  for (const void* ptr : ptrs)
    if (ptr && (reinterpret_cast<uintptr_t>(ptr) % (4 * eb)) != 0) return RB_ERR_UNSUPPORTED;
  // Node K / V rows are staged in shared memory with 16-byte copies: their bases
  // and row / head strides must be whole 16-byte units (8 bf16 or 4 fp32 elements).
  if (nod) {
    const int64_t vec = 16 / eb;
    if (a->sknn % vec || a->svnn % vec || a->sknh % vec || a->svnh % vec ||
        (reinterpret_cast<uintptr_t>(a->kn) & 15) || (reinterpret_cast<uintptr_t>(a->vn) & 15))
      return RB_ERR_UNSUPPORTED;
  }
  return RB_OK;
}

int attn_launch(const rb_attn_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const int st = attn_validate(a);
  if (st != RB_OK) return st;
  if (a->M == 0) return RB_OK;
  const size_t need = attn_workspace_bytes(a->H, a->M, a->D, a->NP);
  if (!ws || ws_bytes < need) return RB_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) & 15) return RB_ERR_UNSUPPORTED;  // partials move by bulk copies
  AttnDev p{};
  p.H = a->H; p.M = a->M; p.HK = a->HK; p.NP = a->NP; p.NN = a->NN;
  p.q = a->q; p.sqh = a->sqh; p.sqm = a->sqm;
  p.kp = a->kp; p.skph = a->skph; p.skpn = a->skpn;
  p.vp = a->vp; p.svph = a->svph; p.svpn = a->svpn;
  p.kn = a->kn; p.sknh = a->sknh; p.sknn = a->sknn;
  p.vn = a->vn; p.svnh = a->svnh; p.svnn = a->svnn;
  p.msk = a->msk; p.mask_kind = a->mask_kind; p.smm = a->smm; p.smn = a->smn;
  p.causal_first = a->causal_first;
  p.out = a->out; p.soh = a->soh; p.som = a->som;
  p.sm_scale = a->sm_scale;
  float* part = static_cast<float*>(ws);
  const int nchunks = prefix_nchunks(a->NP, a->H);
  if (nchunks > 0) {
    if (a->dtype == RB_F32) {  // fp32: three tf32 products per term on the tensor cores (1e-5 parity bar)
      dim3 grid(nchunks, a->H, (a->M + 15) / 16);
      if (cudaFuncSetAttribute(attn_prefix_tf32, cudaFuncAttributeMaxDynamicSharedMemorySize, t32::kSmemBytes) !=
          cudaSuccess)
        return RB_ERR_CUDA;
      attn_prefix_tf32<<<grid, 32 * t32::kWarps, t32::kSmemBytes, stream>>>(p, part);
      if (cudaGetLastError() != cudaSuccess) return RB_ERR_CUDA;
    } else {  // bf16: tcgen05 QK^T / PV with TMA-staged tiles
      CUtensorMap tq, tk, tv;
      if (encode_heads_3d(&tq, a->q, a->M, a->H, a->sqm, a->sqh) != RB_OK ||
          encode_heads_3d(&tk, a->kp, a->NP, a->HK, a->skpn, a->skph) != RB_OK ||
          encode_heads_3d(&tv, a->vp, a->NP, a->HK, a->svpn, a->svph) != RB_OK)
        return RB_ERR_UNSUPPORTED;  // TMA needs 16-byte aligned bases and row strides
      const int st = attn_prefix_tc_launch(tq, tk, tv, p, part, nchunks, stream, false);
      if (st != RB_OK) return st;
    }
  }
  // The node kernel follows under PDL: its folds (q and node K / V only) run
  // beside the prefix kernel, its merges wait for the prefix partials.
  if (a->dtype == RB_F32) return launch_nodes<float>(p, part, stream, nchunks > 0);
  return launch_nodes<uint16_t>(p, part, stream, nchunks > 0);
}

// Engine path: bf16, q/base/PL from device memory, trie masking from the ancestor chains.
int attn_launch_engine(const AttnDev& p, float* part, int max_chunks, const CUtensorMap& tq,
                       const CUtensorMap& tk, const CUtensorMap& tv, cudaStream_t stream) {
  const int st = attn_prefix_tc_launch(tq, tk, tv, p, part, max_chunks, stream, true);
  if (st != RB_OK) return st;
  return launch_nodes<uint16_t>(p, part, stream, true);
}

}  // namespace rb
