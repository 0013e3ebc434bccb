/*
 * hotcold_b200.h — C ABI of the B200 (sm_100a) hot/cold KV decode path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, and returns an
 * HC_* status code; hc_last_error() describes the last failure on the calling
 * thread. Nothing here allocates device memory: callers pass the buffers and a
 * scratch area sized by the *_scratch_bytes() functions.
 *
 * The reference (tarun931/hotcold-kv-cache, src/hotcold_kv) is pure Python with
 * one Triton kernel; each entry point below names the reference function whose
 * behaviour it takes over (file:line in that package).
 *
 * Data layout in HBM, per layer and per sequence (hc_seq_desc):
 *   hot slab   hot_k / hot_v / hot_kpre  [Hk][cap][D]  model dtype
 *              hot_pos [cap] int64, hot_ord [cap] int32 (logical -> physical
 *              slot), hot_free [cap] int32 (stack of free physical slots)
 *   held       held_k / held_v [Hk][r_max][D], held_pos [r_max] int64,
 *              held_valid [r_max] uint8, held_src [r_max] int32 — the retrieved
 *              tokens attended ahead of the hot tokens (post-RoPE keys) and the
 *              cold ring slots they came from
 *   cold ring  cold_vec [ccap][F] float32 index vectors, cold_kpre / cold_v
 *              [ccap][Hk][D] model dtype, cold_pos [ccap] int64
 *   query pool qwin [p_max][D] model dtype: per decode step, the mean over
 *              query heads of the pre-RoPE query
 *   st         device-resident counters (hc_seq_state), updated by kernels.
 */
#ifndef HOTCOLD_B200_H
#define HOTCOLD_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define HC_API __attribute__((visibility("default")))
#else
#define HC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
enum { HC_F32 = 0, HC_F16 = 1, HC_BF16 = 2 };
/* eviction policies */
enum { HC_POLICY_HOTCOLD = 0, HC_POLICY_SNAPKV = 1 };
enum { HC_POOL_MAX = 0, HC_POOL_AVG = 1 };
/* host return codes */
enum { HC_OK = 0, HC_ERR_ARG = 1, HC_ERR_CUDA = 2, HC_ERR_UNSUPPORTED = 3, HC_ERR_SCRATCH = 4 };
/* device status bits (hc_seq_state.status), OR-ed by kernels, cleared by the caller */
enum { HC_DEV_CAPACITY = 1, HC_DEV_TIMEOUT = 2, HC_DEV_INDEX = 4 };

typedef struct hc_seq_state {
  int32_t n_hot;      /* live hot tokens (logical length) */
  int32_t n_free;     /* entries on the free-slot stack */
  int32_t cold_head;  /* ring: physical slot of the oldest live entry */
  int32_t cold_count; /* ring: live entries */
  int32_t held_len;   /* slots of the held segment (lookahead_k once filled) */
  int32_t n_hits;     /* valid hits of the last retrieval: min(R, cold_count) */
  int32_t qwin_head;  /* query pool ring: next write slot */
  int32_t n_evict;    /* tokens evicted by the last compression */
  int32_t status;     /* HC_DEV_* bits */
  int32_t pad[7];
} hc_seq_state;       /* 64 bytes */

typedef struct hc_seq_desc {
  void* hot_k;
  void* hot_v;
  void* hot_kpre;
  int64_t* hot_pos;
  int32_t* hot_ord;
  int32_t* hot_free;
  void* held_k;
  void* held_v;
  int64_t* held_pos;
  uint8_t* held_valid;
  int32_t* held_src;    /* [r_max] cold ring slot of each held entry, -1 = empty */
  float* cold_vec;
  void* cold_kpre;
  void* cold_v;
  int64_t* cold_pos;
  void* qwin;
  hc_seq_state* st;
  int32_t cap;    /* physical hot slots (budget + 1) */
  int32_t budget; /* max_capacity_prompt of this sequence */
  int32_t r_max;  /* held slots (lookahead_k) */
  int32_t ccap;   /* cold ring capacity (cpu_buffer_size) */
  int32_t p_max;  /* query pool capacity (query_pool_size) */
  int32_t pad[1];
} hc_seq_desc;    /* 160 bytes */

/* One layer: n_seq sequences sharing head geometry and policy knobs. */
typedef struct hc_layer {
  const hc_seq_desc* desc; /* device array [n_seq] */
  const float* inv_freq;   /* device [D/2] rotary inverse frequencies */
  int32_t* counters;       /* device [n_seq*Hk] int32, zero before first use; kernels leave it zero */
  double topk_ratio;       /* hot/cold policy: prefix share of the budget, int(budget*topk_ratio) */
  int32_t n_seq;
  int32_t Hq, Hk, D;       /* query heads, KV heads, head dim (D in {64,128}) */
  int32_t F;               /* index vector length (faiss_dim) */
  int32_t dtype;           /* HC_F32 / HC_F16 / HC_BF16 */
  int32_t policy;          /* HC_POLICY_* */
  int32_t recent;          /* recent_size (SnapKV: observation/recent window) */
  int32_t pool_kernel;     /* SnapKV pooling width (odd) */
  int32_t pooling;         /* HC_POOL_* */
  int32_t normalize;       /* L2-normalise index and query vectors */
  int32_t max_cap;         /* max hot slots over sequences */
  int32_t max_r;           /* max held slots over sequences */
  int32_t max_ccap;        /* max cold ring capacity over sequences */
  float scale;             /* attention scale, 1/sqrt(D) */
  float rope_scaling;      /* rotary attention_scaling */
  const void* kmaps;       /* optional device array of four 128-byte TMA tensor maps written by
                              hc_encode_kmap (f16/bf16), each over all sequences as rows of D
                              elements: [0] the hot K slab, box 64 x 64 rows; [1] the held K
                              rows, box 64 x 8 rows; [2] the hot V slab, box 64 x 16 rows; [3]
                              the held V rows, box 64 x 8 rows. hc_step needs them for 16-bit
                              dtypes. */
} hc_layer;                /* 104 bytes */

/* Library and error reporting. */
HC_API const char* hc_version(void);

/*
 * The device address of page-locked host memory (cudaHostGetDevicePointer): where a cold ring's
 * payload lives in host RAM (KVController(cold_payload="host"); no counterpart in the reference,
 * whose cold tier is host memory that the GPU never reads directly), the descriptors point
 * the kernels at it. HC_ERR_ARG when `host` is not page-locked memory known to CUDA.
 */
HC_API int hc_host_device_pointer(const void* host, void** dev);
HC_API const char* hc_last_error(void);

/*
 * Stand-alone decode attention over dense K/V, the drop-in for
 * triton_evict_attention_forward (kernels.py:77-137; kernel kernels.py:9-74).
 * q (B,Hq,D), k/v (B,Hk,S,D), mask (B,S) uint8 (nonzero = attend), all
 * contiguous; out (B,Hq,D) in the input dtype. With evict_idx non-null it also
 * writes the wrapper's second result: argmin over tokens of the head-mean of
 * softmax(q.k) * sum|v|/D, cast to the input dtype (kernels.py:134-137).
 * overflow_nan=1 reproduces the reference's unstabilised exp: a head whose
 * largest unmasked logit overflows fp32 exp yields NaN.
 */
HC_API size_t hc_attention_dense_scratch_bytes(int B, int Hq, int Hk, int S, int D);
HC_API int hc_attention_dense(const void* q, const void* k, const void* v, const uint8_t* mask, void* out,
                       int64_t* evict_idx, int B, int Hq, int Hk, int S, int D, int dtype, float scale,
                       int overflow_nan, int32_t* counters, void* scratch, size_t scratch_bytes,
                       void* stream);

/*
 * hc_attention_dense for callers that cannot allocate device memory (no
 * counterpart in the reference): a host that binds this library over FFI and
 * passes only its inputs and outputs, or a process whose device memory is all
 * reserved by its own pool. Scratch and counters live in static device arrays
 * of the library (8 MiB + 4096 counters, held on every GPU that loads it until
 * exit); shapes needing more are rejected with HC_ERR_UNSUPPORTED. Calls share
 * those arrays, so calls that overlap on the GPU race. Every call resolves the
 * arrays' addresses on the current device. Under lazy module loading (the CUDA
 * 12.x default) the arrays are committed when the first call on a device loads
 * the module: make that call before the caller's pool reserves the device's
 * memory and before any stream capture, or set CUDA_MODULE_LOADING=EAGER.
 * Allocates nothing: no cudaMalloc/cudaFree.
 */
HC_API int hc_attention_dense_noalloc(const void* q, const void* k, const void* v, const uint8_t* mask, void* out,
                                      int64_t* evict_idx, int B, int Hq, int Hk, int S, int D, int dtype,
                                      float scale, int overflow_nan, void* stream);

/*
 * Decode-step append: RoPE of the new query/key with the model's cos/sin
 * (patch.py:161-162), append of (k_post, v, k_pre, pos) to the hot slab
 * (HotColdLayer.update, cache.py:130-151) and push of the head-mean query to
 * the query pool (KVController.update_query_window, controller.py:240-241).
 * q_pre (n_seq,Hq,D), k_pre/v (n_seq,Hk,D) with row strides in elements;
 * cos/sin (n_seq,D) in the model dtype, or NULL to compute them from
 * inv_freq and pos; q_post out (n_seq,Hq,D) contiguous.
 */
HC_API int hc_append(const hc_layer* L, const void* q_pre, int64_t q_stride_seq, const void* k_pre,
              const void* v, int64_t kv_stride_seq, const void* cos, const void* sin,
              const int64_t* pos, void* q_post, void* stream);

/*
 * Append of already-rotated keys (the HotColdLayer.update entry, cache.py:130-151):
 * k_post/k_pre/v (n_seq,Hk,D) with row stride kv_stride_seq, no query.
 */
HC_API int hc_append_rotated(const hc_layer* L, const void* k_post, const void* k_pre, const void* v,
                      int64_t kv_stride_seq, const int64_t* pos, void* stream);

/*
 * Append evicted tokens to the cold ring and index (add_evicted_to_cold_store,
 * controller.py:190-238): k_pre/v (n_seq,Hk,Te,D) with strides (seq, head,
 * token) in elements, pos and evicted_idx (n_seq,Te) int64; entries with
 * evicted_idx < 0 are skipped; a batch larger than the ring keeps its newest
 * ccap tokens.
 */
HC_API int hc_cold_append(const hc_layer* L, const void* k_pre, const void* v, int64_t s_seq, int64_t s_head,
                   int64_t s_tok, const int64_t* pos, const int64_t* evicted_idx, int Te, void* stream);

/*
 * Compression of the hot tier (HotColdLayer._compress_if_needed,
 * cache.py:37-128; SnapKV scoring scoring.py:50-79 with keep_index
 * scoring.py:110-132 under HC_POLICY_SNAPKV), with the evicted tokens appended
 * to the cold ring and its index (add_evicted_to_cold_store,
 * controller.py:190-238). q_obs (n_seq,Hq,tq,D) holds the post-RoPE
 * observation queries (strides in elements); the last min(tq, window) rows
 * are used. Each sequence computes its own plan from its length S and budget
 * (cache.py:44-53 / scoring.py:117-120) and does nothing when S <= budget.
 * Source:
 *   src_k == NULL: the hot slab itself, S = st->n_hot (decode; S_dense ignored);
 *   otherwise dense prompt tensors src_k/src_v/src_kpre (n_seq,Hk,S_dense,D)
 *   with strides (seq, head, token) in elements and src_pos (n_seq,S_dense)
 *   int64 on an empty slab (prefill); kept tokens are copied into the slab.
 */
HC_API size_t hc_compress_scratch_bytes(const hc_layer* L, int S_max, int tq);
HC_API int hc_compress(const hc_layer* L, const void* q_obs, int64_t qs_seq, int64_t qs_head, int64_t qs_tok,
                int tq, int S_dense, const void* src_k, const void* src_v, const void* src_kpre,
                int64_t ss_seq, int64_t ss_head, int64_t ss_tok, const int64_t* src_pos, void* scratch,
                size_t scratch_bytes, void* stream);

/*
 * hc_compress with a launch hint: n_evict_hint is the largest number of tokens
 * any sequence evicts in this call (the host can compute it from the same
 * plan). Evictions of at most 32 tokens are copied by the selection CTA
 * itself; a larger hint adds the multi-CTA copy kernel. The hint must not be
 * below the true count; hc_compress passes "unknown" (always add the kernel).
 */
HC_API int hc_compress_ex(const hc_layer* L, const void* q_obs, int64_t qs_seq, int64_t qs_head, int64_t qs_tok,
                   int tq, int S_dense, const void* src_k, const void* src_v, const void* src_kpre,
                   int64_t ss_seq, int64_t ss_head, int64_t ss_tok, const int64_t* src_pos, void* scratch,
                   size_t scratch_bytes, int n_evict_hint, void* stream);

/*
 * Prefill store without compression (S <= budget): copy the prompt into the
 * hot slab in order (cache.py:145-148 on an empty cache).
 */
HC_API int hc_store_prompt(const hc_layer* L, int S, const void* src_k, const void* src_v, const void* src_kpre,
                    int64_t ss_seq, int64_t ss_head, int64_t ss_tok, const int64_t* src_pos, void* stream);

/*
 * Retrieval: pooled query vector (_q_to_vecs_np / _pooled_query_np,
 * controller.py:184-188,243-248), exact inner-product top-R over the cold
 * index (IndexFlatIP.search, controller.py:274; ties to the older entry),
 * gather of the hits (controller.py:277-285), RoPE at their original positions
 * (_rotate_k_with_pos, patch.py:94-102) and splice into the held segment
 * (patch.py:249-256). Query source: q_dense != NULL gives pre-RoPE queries
 * (n_seq,Hq,P,D) with strides (seq, head, token) — the prompt tail of
 * launch_retrieval_now (patch.py:232); otherwise the newest n_pool entries of
 * the query pool, plus an optional fp32 prompt-query sum `extra_sum`
 * (n_seq,D) covering `extra_n` positions (query_pool_size >= window_size keeps
 * the prompt queries in the pool, patch.py:169-170).
 */
HC_API size_t hc_retrieve_scratch_bytes(const hc_layer* L);
HC_API int hc_retrieve(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head, int64_t qd_tok,
                int P, int n_pool, const float* extra_sum, int extra_n, void* scratch, size_t scratch_bytes,
                void* stream);

/*
 * hc_retrieve with a grid hint and an optional given query: max_count bounds
 * the live cold entries of any sequence (0 = the ring capacity), which sizes
 * the scan grid; qvec_in (n_seq,F) fp32, when non-NULL, is searched as is
 * (the q_vecs argument of _retrieval_worker, controller.py:250).
 */
HC_API int hc_retrieve_ex(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head, int64_t qd_tok, int P,
                   int n_pool, const float* extra_sum, int extra_n, const float* qvec_in, void* scratch,
                   size_t scratch_bytes, int max_count, void* stream);

/*
 * Head-mean prompt queries summed over positions, fp32 (n_seq,D): the prompt's
 * contribution to the query pool when it stays in the pool (update_query_window,
 * controller.py:240-241, with the pooled mean of controller.py:243-248). Scratch
 * from hc_prompt_query_sum_scratch_bytes (per-CTA partial sums).
 */
HC_API size_t hc_prompt_query_sum_scratch_bytes(const hc_layer* L);
HC_API int hc_prompt_query_sum(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head,
                        int64_t qd_tok, int P, float* out_sum, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Decode attention over [held | hot] (patch.py:263-305 and the Triton kernel
 * kernels.py:9-74): held slot j attends iff held_valid[j] and
 * held_pos[j] <= cur_pos (patch.py:287-289), hot tokens always. q_post
 * (n_seq,Hq,D) contiguous, cur_pos (n_seq) int64, out (n_seq,Hq,D).
 */
HC_API size_t hc_attend_scratch_bytes(const hc_layer* L);
HC_API int hc_attend(const hc_layer* L, const void* q_post, const int64_t* cur_pos, int use_held, void* out,
              int overflow_nan, void* scratch, size_t scratch_bytes, void* stream);

/*
 * Decode-step retrieval whose pooled query is this step's pre-RoPE query q_pre
 * (n_seq, Hq, D) with sequence stride q_stride_seq, taken as the newest pool entry (the mean
 * over its heads rounded to the dtype, as the query-pool push computes it), followed by the
 * n_pool newest entries of the query pool: the search of controller.py:314-342 for a step
 * whose query-pool push happens later in hc_step. Search, gather and re-RoPE into the held
 * segment as hc_retrieve. No counterpart in the reference (its push precedes the search in
 * the same Python call). Returns HC_ERR_UNSUPPORTED when the fused retrieval kernel does not
 * fit the layer.
 */
HC_API int hc_retrieve_decode(const hc_layer* L, const void* q_pre, int64_t q_stride_seq, int n_pool, void* scratch,
                              size_t scratch_bytes, void* stream);

/*
 * TMA tensor map for hc_layer.kmaps, encoded on the host into `out` (128 bytes, copy it to
 * 64-byte aligned device memory): a 2-D map over `rows` rows of D elements of dtype
 * (HC_F16 or HC_BF16) starting at device address `base` (16-byte aligned, rows contiguous),
 * box 64 elements x box_rows rows (1..256), 128-byte swizzle, out-of-range rows read as
 * zero. No counterpart in the reference: it serves the TMA loads of the fused step.
 * Returns HC_ERR_UNSUPPORTED when the driver offers no tensor-map encoder.
 */
HC_API int hc_encode_kmap(void* out, const void* base, int dtype, int64_t rows, int D, int box_rows);

/*
 * Whether hc_step would launch for this layer (HC_OK) or return HC_ERR_UNSUPPORTED, checked
 * without launching anything. No counterpart in the reference: it lets a caller decide
 * between the fused step and the split ops before starting a step.
 */
HC_API int hc_step_check(const hc_layer* L, int use_held);

/*
 * Fused decode step of one layer: hc_append, hc_compress (decode, slab source)
 * and hc_attend in one launch (patch.py:151-305 with cache.py:37-151 and the
 * kernel of kernels.py:9-74), one 16-CTA thread-block cluster per sequence
 * (CTA = KV head x token part). Same arguments and results as the three calls
 * in sequence; out (n_seq,Hq,D). Returns HC_ERR_UNSUPPORTED (nothing launched)
 * when the layer does not fit one cluster; callers then use the three calls.
 *
 * The kernel is launched with programmatic stream serialisation: it may start
 * while the launch before it on the stream still runs, and waits for that
 * launch before it reads the step's inputs. `early` lets it read part of this
 * layer's state before that wait, overlapping those copies with the preceding
 * launch. The caller sets a bit only when that launch writes none of the state
 * the bit names: HC_STEP_EARLY_HOT the hot slab rows, logical order and free
 * stack (true after another layer's step or this layer's hc_retrieve_decode);
 * HC_STEP_EARLY_HELD the held segment (not after this layer's retrieval). 0 is
 * always correct.
 */
#define HC_STEP_EARLY_HOT 1
#define HC_STEP_EARLY_HELD 2
HC_API int hc_step(const hc_layer* L, const void* q_pre, int64_t q_stride_seq, const void* k_pre, const void* v,
                   int64_t kv_stride_seq, const void* cos, const void* sin, const int64_t* pos, int use_held,
                   void* out, int overflow_nan, int early, void* stream);

/*
 * Multi-GPU cold search over a token-range shard: merge of per-shard top-k
 * candidates gathered from all ranks (no reference counterpart; the reference
 * is single-device). cand_score/cand_id (n_shards*k) fp32/int32, global ids;
 * writes the global top-k ids (ties to the lower id), sorted by score.
 */
HC_API int hc_shard_merge(const float* cand_score, const int32_t* cand_id, int n_shards, int k, int32_t* out_id,
                   float* out_score, void* stream);

/*
 * Exact inner-product top-k over n_rows index vectors (row-major fp32, F per row): the
 * IndexFlatIP.search of controller.py:274 over one block of the cold index, e.g. the
 * token-range shard a rank holds. qvec (F) fp32 on the device; writes the k best as
 * (out_score, out_id) sorted by score, ids id_base + row, ties to the lower id, -1 / -inf
 * past n_rows. Rows are scored with the ring scan's arithmetic, so a row's score does not
 * depend on the block it sits in. Scratch from hc_cold_topk_scratch_bytes.
 */
HC_API size_t hc_cold_topk_scratch_bytes(int64_t n_rows, int k);
HC_API int hc_cold_topk(const float* index, int64_t n_rows, int F, int64_t id_base, const float* qvec, int k,
                        float* out_score, int32_t* out_id, void* scratch, size_t scratch_bytes, void* stream);

/*
 * The pooled query vector of hc_retrieve alone (_q_to_vecs_np / _pooled_query_np,
 * controller.py:184-188,243-248; same query sources and rounding), written to out_qvec
 * (n_seq, F) fp32: the query a sharded search hands to hc_cold_topk.
 *
 * Held segment from given hits: hit_ids (n_seq, k) int32 are live cold entries in age order
 * (0 = the oldest live entry, the numbering of the cold ring's index), -1 for none. Slot j
 * takes hit j: gather of the payload (controller.py:277-285), RoPE at the original position
 * (patch.py:94-102) and splice (patch.py:249-256), as the tail of hc_retrieve. Used after a
 * search done elsewhere (hc_cold_topk on index shards and hc_shard_merge).
 */
HC_API int hc_retrieve_query(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head,
                             int64_t qd_tok, int P, int n_pool, const float* extra_sum, int extra_n, float* out_qvec,
                             void* stream);
HC_API int hc_splice_hits(const hc_layer* L, const int32_t* hit_ids, int k, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HOTCOLD_B200_H */
