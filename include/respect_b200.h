/*
 * respect_b200 — C ABI of the B200-native trie-verify hot path of RESPECT
 * (soonhong99/respect).
 *
 * Every entry point takes caller-owned device pointers, sizes and strides (in
 * elements) plus a cudaStream_t passed as `void*`, launches asynchronously on
 * that stream and returns an rb_status code. None of them allocates device
 * memory: kernels that need scratch take a caller-provided workspace whose size
 * the matching *_workspace() query returns. No torch types cross this boundary.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   rb_fused_attn_hyb   respect/kernels/attention.py:74-96   fused_attn_hyb
 *   rb_linear           respect/kernels/gemm.py:30-41        linear
 *   rb_rmsnorm          respect/kernels/rmsnorm.py:25-32     rmsnorm
 *   rb_rope             respect/system/fused.py:67-75        rope
 *   rb_silu_mul         respect/system/fused.py:116-123      silu_mul
 *   rb_add_sq, rb_norm_apply  respect/system/fused.py:126-194 add_sq / norm_from (Prefill)
 *   rb_linear_swiglu_packed  fused.py:106-123 silu_mul fused into the gate|up linear (patch.py:26-37)
 *   rb_greedy_token     respect/decoding/acceptance.py:11-23 mask_action_vocab + greedy_token
 *   rb_compact_kv       respect/decoding/kv_buffer.py:93-104 compact
 *   rb_trie_node_mask   respect/candidates/trie.py:51-64 + respect/kernels/dispatch.py:94-115
 *   rb_verify_mask      respect/decoding/verify.py:35-41     additive 4-D trie mask
 *   rb_engine_*         respect/decoding/verify.py:12-46 + respect/kernels/patch.py:70-107
 *                       (one verify forward of the whole decoder with the dedicated kernels)
 *   rb_engine_accept    respect/decoding/acceptance.py:26-46 + kv_buffer.py:93-104 on the device
 */
#ifndef RESPECT_B200_H
#define RESPECT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RB_ABI_VERSION 1

#if defined(__GNUC__)
#define RB_API __attribute__((visibility("default")))
#else
#define RB_API
#endif

/* Status codes returned by every entry point. */
enum rb_status {
  RB_OK = 0,
  RB_ERR_INVALID_ARG = 1,    /* null pointer, negative size, bad stride */
  RB_ERR_UNSUPPORTED = 2,    /* shape / dtype / layout this build does not handle */
  RB_ERR_CAPACITY = 3,       /* size beyond a fixed limit (rows, nodes, buffer slots) */
  RB_ERR_CUDA = 4,           /* a CUDA runtime / driver call failed */
  RB_ERR_DEVICE_TIMEOUT = 5, /* a bounded device-side wait gave up (see rb_device_error) */
  RB_ERR_WORKSPACE = 6       /* workspace missing or smaller than *_workspace() */
};

/* Element types. */
enum rb_dtype { RB_F32 = 0, RB_BF16 = 1, RB_U8 = 2, RB_I32 = 3, RB_I64 = 4 };

/* How rb_fused_attn_hyb reads the node mask. */
enum rb_mask_kind {
  RB_MASK_BOOL = 0,   /* uint8 [M, NN]: nonzero = attend (the reference's bool msk) */
  RB_MASK_ADD_BF16 = 1, /* bf16 additive [M, NN]: attend iff value == 0 (dispatch.py:141-143) */
  RB_MASK_ADD_F32 = 2,  /* fp32 additive [M, NN]: attend iff value == 0 */
  RB_MASK_CAUSAL = 3    /* no buffer: row r attends node j iff j <= r + causal_first (dispatch.py:206-210) */
};

RB_API const char* rb_status_string(int status);
RB_API int rb_abi_version(void);
RB_API int rb_num_sms(void);

/* Device-side error flag set by a bounded wait that gave up (0 = none).
 * Reading it synchronises the current device. */
RB_API int rb_device_error(int* code, int clear);

/* ------------------------------------------------------------------ attention
 * Trie-verification attention (respect/kernels/attention.py:15-96).
 * q [H, M, D], kp/vp [HK, NP, D] (prefix, no mask), kn/vn [HK, NN, D] (node
 * slots), msk per rb_mask_kind, out [H, M, D]. GQA: head h reads kv head
 * h / (H / HK). The prefix is reduced in fixed 128-key tiles grouped into
 * fixed chunks at absolute key positions, combined in chunk order; node slots
 * are accumulated one at a time in slot order and masked slots are skipped, so
 * a row's result depends only on its own allowed keys and their order. All
 * accumulation is fp32, the output is cast once.
 * Innermost strides (sqd, skpd, ...) must be 1. dtype RB_F32 or RB_BF16.
 * Layout limits (RB_ERR_UNSUPPORTED otherwise): D = 128; other strides in
 * multiples of 4 elements and bases aligned to 4 elements; kp / vp (bf16) and
 * kn / vn (both dtypes) in whole 16-byte rows: strides and bases multiples of
 * 16 bytes. */
typedef struct rb_attn_args {
  int dtype;
  int H, M, D, HK, NP, NN;
  const void* q;  int64_t sqh, sqm, sqd;
  const void* kp; int64_t skph, skpn, skpd;
  const void* vp; int64_t svph, svpn, svpd;
  const void* kn; int64_t sknh, sknn, sknd;
  const void* vn; int64_t svnh, svnn, svnd;
  const void* msk; int mask_kind; int64_t smm, smn;
  int causal_first;
  void* out; int64_t soh, som, sod;
  float sm_scale;
} rb_attn_args;

RB_API size_t rb_fused_attn_hyb_workspace(int H, int M, int D, int NP);
RB_API int rb_fused_attn_hyb(const rb_attn_args* a, void* workspace, size_t ws_bytes, void* stream);

/* The same attention for callers that cannot allocate device memory (no
 * cudaMalloc allowed where they run, or only their inputs and outputs in hand):
 * the scratch lives in a 16 MiB array of device memory owned by the library, one
 * per GPU that loads it, kept until the process exits. This entry point itself
 * allocates nothing. No counterpart in the reference (its Triton kernel needs
 * no scratch).
 *  - Calls needing more than 16 MiB of scratch (rb_fused_attn_hyb_workspace)
 *    return RB_ERR_CAPACITY.
 *  - The array's address is looked up in the caller's current CUDA context the
 *    first time the entry point runs there (a primary context, a context the
 *    caller created, a context re-created after a device reset); make that first
 *    call before capturing a stream into a CUDA graph.
 *  - All calls share the one array: calls that may overlap on the GPU (different
 *    streams, concurrent graphs) race on it and must be serialised by the caller.
 *  - The array keeps the last call's contents; nothing in it needs to start at zero. */
RB_API int rb_fused_attn_hyb_noalloc(const rb_attn_args* a, void* stream);

/* ------------------------------------------------------------------ linear
 * out[M, N] = x[M, K] @ w[N, K]^T with a row-count-invariant reduction
 * (respect/kernels/gemm.py:11-41). x, w bf16 with unit inner stride; out
 * RB_BF16 or RB_F32 (the lm_head case, respect/kernels/patch.py:23). K % 8 == 0,
 * row strides % 8 == 0, pointers 16-byte aligned. */
RB_API size_t rb_linear_workspace(int M, int N, int K);
RB_API int rb_linear(const void* x, int64_t ldx, const void* w, int64_t ldw, void* out, int64_t ldo,
              int out_dtype, int M, int N, int K, void* workspace, size_t ws_bytes, void* stream);

/* Packed weights for the weight-streaming GEMM: [ceil(N/BN)][ceil(K/64)][BN][64]
 * bf16 (zero padded), so each pipeline stage reads one contiguous block. BN is
 * the tile width rb_linear chooses for (N, K) (rb_linear_bn); BN <= 0 selects
 * it. rb_linear_packed gives bitwise the same result as rb_linear on the
 * unpacked weight (same MMA sequence per output element). No reference
 * counterpart: a storage layout of the same linear (gemm.py:30-41). */
RB_API int rb_linear_bn(int N, int K);
RB_API size_t rb_linear_packed_bytes(int N, int K, int BN);
RB_API int rb_pack_linear_weight(const void* w, int64_t ldw, int N, int K, int BN, void* out, void* stream);
RB_API int rb_linear_packed(const void* x, int64_t ldx, const void* w_packed, void* out, int64_t ldo,
                            int out_dtype, int M, int N, int K, void* workspace, size_t ws_bytes, void* stream);

/* Fused SwiGLU projection: out[M, F] = silu(x Wg^T) * (x Wu^T), bf16, the HF MLP's
 * act_fn(gate_proj(x)) * up_proj(x) with its rounding points (each projection
 * rounded to bf16, silu rounded, product rounded; respect/system/fused.py:106-123
 * on top of the dedicated linears of respect/kernels/patch.py:26-37), in one
 * launch: the SiLU*mul runs in the GEMM epilogue, the two projections never
 * reach HBM. w_gu is Wg and Wu [F, K] interleaved in 128-row blocks (rows
 * 256i..256i+127 = Wg rows 128i.., rows 256i+128.. = Wu rows 128i..), packed by
 * rb_pack_linear_weight(N = 2F, BN = 256). One K split at every shape, so a
 * row's result does not depend on M; where rb_linear's own plan for (2F, K) is
 * also one split of 256-wide tiles (F = 18944, K = 3584, for one), it is bitwise
 * equal to rb_linear_packed on that weight followed by rb_silu_mul on the two
 * halves. F % 128 == 0; no workspace. */
RB_API int rb_linear_swiglu_packed(const void* x, int64_t ldx, const void* w_gu, void* out, int64_t ldo, int M,
                                   int F, int K, void* stream);

/* ------------------------------------------------------------------ rmsnorm
 * y = w * to_dtype(x * rsqrt(mean(x^2) + eps)), one row per block, fixed
 * reduction order (respect/kernels/rmsnorm.py:12-32). x, y contiguous [M, N]. */
RB_API int rb_rmsnorm(const void* x, const void* w, void* y, int M, int N, float eps, int x_dtype,
               int w_dtype, void* stream);

/* ------------------------------------------------------------------ rope
 * y = x*cos + rotate_half(x)*sin with PyTorch's rounding points: every op
 * rounded to bf16 when the output is bf16, fp32 otherwise; no FMA contraction
 * (respect/system/fused.py:45-75). x [B, H, L, D] strided, cos/sin [B, L, D]
 * (strides scb, scl; unit inner stride), y contiguous [B, H, L, D]. */
RB_API int rb_rope(const void* x, int64_t sxb, int64_t sxh, int64_t sxl, int64_t sxd, const void* cos,
            const void* sin, int64_t scb, int64_t scl, void* y, int B, int H, int L, int D,
            int x_dtype, int cs_dtype, int y_dtype, void* stream);

/* ------------------------------------------------------------------ silu_mul
 * dtype RB_BF16: y = bf16(bf16(g / (1 + exp(-g))) * u) (respect/system/fused.py:106-123);
 * dtype RB_F32: y = (g / (1 + exp(-g))) * u in fp32 (the reference's eager
 * branch for non-bf16 inputs, fused.py:117-118). Contiguous, n elements. */
RB_API int rb_silu_mul(const void* g, const void* u, void* y, int64_t n, int dtype, void* stream);

/* ------------------------------------------------------------------ prefill norm pieces
 * respect/system/fused.py:126-194 (add_sq, norm_from): the elementwise parts of
 * an eager residual add + RMSNorm, bit for bit, around the row mean of squares
 * that the caller computes with PyTorch. rb_add_sq: x = r + h in the promoted
 * dtype (bf16 only when both are bf16), sq = x * x in fp32; h = NULL gives
 * sq = r * r alone (x unused). rb_norm_apply: y = w * to_x_dtype(x * rsqrt(var
 * + eps)), var [M] fp32, y in promote(w, x). Contiguous [M, N] / [n] tensors. */
RB_API int rb_add_sq(const void* r, const void* h, void* x, float* sq, int64_t n, int r_dtype, int h_dtype,
                     int x_dtype, void* stream);
RB_API int rb_norm_apply(const void* x, const float* var, const void* w, void* y, int64_t M, int N, float eps,
                         int x_dtype, int w_dtype, int y_dtype, void* stream);

/* ------------------------------------------------------------------ greedy token
 * out[m] = argmax_v logits[m, v] with v in [offset, offset + size) excluded;
 * ties resolve to the lowest index (acceptance.py:11-23). logits RB_F32 or RB_BF16. */
RB_API int rb_greedy_token(const void* logits, int dtype, int64_t ld, int M, int V, int offset, int size,
                    int64_t* out, void* stream);

/* ------------------------------------------------------------------ compact
 * For every layer and both K and V: slot dst_start + i <- slot src_slots[i]
 * (kv_buffer.py:93-104). Each cache tensor is [HK, S, D] with strides
 * (s_head, s_slot, 1); src_slots are absolute slot numbers, strictly
 * increasing with src_slots[i] >= dst_start + i (an accepted trie path).
 * Up to RB_COMPACT_MAX_LAYERS layers and RB_COMPACT_MAX_SLOTS slots. */
#define RB_COMPACT_MAX_LAYERS 128
#define RB_COMPACT_MAX_SLOTS 1024
RB_API int rb_compact_kv(void* const* k_layers, void* const* v_layers, int n_layers, int HK, int D,
                  int64_t s_head, int64_t s_slot, int elem_bytes, const int32_t* src_slots, int n,
                  int dst_start, void* stream);

/* ------------------------------------------------------------------ trie masks
 * parents: device int32 [q], parents[i] < i or -1 for a root (trie.py:31-48
 * insertion order). rb_trie_node_mask writes the kernel's bool node mask
 * msk[M, NN] (row stride ld): row i < q opens the `committed` slots before the
 * trie and the ancestors-or-self of node i (trie.py:51-64); rows q..M-1 open
 * slot 0 only (dispatch.py:115); every other entry is 0.
 * rb_verify_mask writes verify.py's additive bf16 mask m[q, width]: 0 for
 * columns < start and for trie ancestors-or-self at start + j, bf16 lowest
 * elsewhere. */
RB_API int rb_trie_node_mask(const int32_t* parents, int q, int committed, int M, int NN, uint8_t* msk,
                      int64_t ld, void* stream);
RB_API int rb_verify_mask(const int32_t* parents, int q, int start, int width, void* mask_bf16,
                   void* stream);

/* ------------------------------------------------------------------ verify engine
 * One verify forward of a Qwen3-style decoder over the nodes of a trie, with
 * the dedicated kernels (respect/decoding/verify.py:12-46 run through HF with
 * respect/kernels/patch.py:70-107 installed), composed natively: embedding,
 * L x [RMSNorm, q|k|v linear, per-head q/k RMSNorm, RoPE, KV write, trie
 * attention, o linear, residual, RMSNorm, gate|up linear, SiLU*mul, down
 * linear, residual], final RMSNorm, fp32 lm_head, greedy choice with the
 * action-vocabulary range excluded (acceptance.py:11-23).
 *
 * Node i of a step is written to KV slot prompt_len + base + i and rotated at
 * position prompt_len + base + depth[i] + rope_delta (verify.py:24-33); it
 * attends to the prefix [0, prompt_len), the `base` committed slots, and its
 * own trie ancestors-or-self (verify.py:35-41). Step values live in device
 * memory, so one CUDA graph per power-of-two row bucket serves every step.
 * Weights, KV buffers and the workspace are caller-owned device memory; the
 * engine never calls cudaMalloc (creation allocates a small pinned host
 * staging buffer; graph instantiation lets the runtime allocate its own
 * resources). */
typedef struct rb_model_config {
  int hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab;
  float rms_eps;
  int max_rows;  /* largest trie (query rows) of a step, <= 1024 */
  int max_slots; /* slots of every per-layer KV buffer: prompt + capacity */
  int max_pos;   /* rows of the rotary tables */
} rb_model_config;

/* Per layer, bf16 device pointers. The four projection matrices are given in
 * the packed layout of rb_pack_linear_weight (BN = rb_linear_bn(N, K), except
 * wgu: BN = 256) of these logical [N, K] matrices:
 *   wqkv [(n_heads + 2 n_kv_heads) * 128, hidden]   q_proj | k_proj | v_proj rows
 *   wo   [hidden, n_heads * 128]
 *   wgu  [2 ffn, hidden]  gate_proj and up_proj interleaved in 128-row blocks:
 *        rows [256 b, 256 b + 128) = gate rows [128 b, 128 b + 128),
 *        rows [256 b + 128, 256 b + 256) = up rows [128 b, 128 b + 128)
 *   wd   [hidden, ffn]
 *   in_norm, post_norm [hidden]; q_norm, k_norm [128] (plain vectors) */
typedef struct rb_layer_weights {
  const void *wqkv, *wo, *wgu, *wd, *in_norm, *post_norm, *q_norm, *k_norm;
} rb_layer_weights;

/* embed [vocab, hidden] bf16 (row-major), lm_head [vocab, hidden] bf16 packed
 * (rb_pack_linear_weight, BN = rb_linear_bn(vocab, hidden)); final_norm [hidden] bf16; rope_cos /
 * rope_sin [max_pos, 128] bf16 (the model's rotary table cast to bf16);
 * layers: host array of n_layers; k_cache / v_cache: host arrays of n_layers
 * device buffers, each [n_kv_heads, max_slots, 128] bf16 contiguous. */
typedef struct rb_model_weights {
  const void* embed;
  const void* final_norm;
  const void* lm_head;
  const void* rope_cos;
  const void* rope_sin;
  const rb_layer_weights* layers;
  void* const* k_cache;
  void* const* v_cache;
} rb_model_weights;

typedef struct rb_engine rb_engine;

/* One step: q trie nodes (ids, parents with parents[i] < i or -1, depths),
 * `base` committed tokens after a `prompt_len`-token prefix. host_inputs = 1:
 * the three arrays are host memory (validated, staged through pinned memory
 * and copied on `stream`); 0: device memory. use_graph = 1 replays the CUDA
 * graph of the row bucket (captured on first use; the first step of a bucket
 * must not run under a caller's stream capture). */
typedef struct rb_step_desc {
  int q, base, prompt_len, rope_delta, act_off, act_size;
  const int32_t* ids;
  const int32_t* parents;
  const int32_t* depths;
  int host_inputs;
  int use_graph;
} rb_step_desc;

RB_API size_t rb_engine_workspace_bytes(const rb_model_config* cfg);
RB_API int rb_engine_create(const rb_model_config* cfg, const rb_model_weights* w, void* workspace,
                            size_t ws_bytes, rb_engine** out);
RB_API int rb_engine_destroy(rb_engine* e);
RB_API int rb_engine_step(rb_engine* e, const rb_step_desc* d, void* stream);
/* Device pointers of the last step's outputs: logits fp32 [bucket, vocab]
 * (rows < q valid), greedy ids int64 [q], residual stream bf16 [bucket, hidden]. */
RB_API int rb_engine_outputs(rb_engine* e, float** logits, int64_t** next_ids, void** hidden, void** reserved);
/* Async copy of the first n greedy ids to host memory on `stream`. */
RB_API int rb_engine_fetch_ids(rb_engine* e, int64_t* host, int n, void* stream);
/* kv_buffer.py:93-104 for every layer: slots prompt_len + base + path[i] move
 * to prompt_len + base + i (path = accepted node indices, host array). */
RB_API int rb_engine_compact(rb_engine* e, const int32_t* path, int n, int prompt_len, int base, void* stream);
/* The acceptance walk (acceptance.py:26-46) and the compaction (kv_buffer.py:93-104)
 * of the last step on the device, without a host round trip: from the step's
 * trie and greedy picks, the accepted chain (root holding `first`, each next
 * node holding the pick after its parent, stopping after `eos` or `cap` tokens)
 * is recorded and its KV moved to slots prompt_len + base + i. Enqueue on the
 * step's stream after rb_engine_step. rb_engine_fetch_accept copies the record
 * to host as [count, correction, base, prompt_len, path[0..n), tokens[0..n)]
 * (count <= n needs n >= the trie size or >= cap). */
RB_API int rb_engine_accept(rb_engine* e, int first, int cap, int eos, void* stream);
RB_API int rb_engine_fetch_accept(rb_engine* e, int32_t* host, int n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RESPECT_B200_H */
