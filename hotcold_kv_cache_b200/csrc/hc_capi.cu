// C ABI of the hot/cold decode path: argument checks, scratch carving, launches.
// Declarations and the reference function each entry replaces: include/hotcold_b200.h.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "hc_internal.cuh"


namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return HC_OK;
  // a rejected launch leaves the runtime's last-error set; clear it so the caller's next,
  // unrelated CUDA call does not report it
  (void)cudaGetLastError();
  return fail(HC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_layer(const hc_layer* L) {
  if (!L || !L->desc) return fail(HC_ERR_ARG, "layer or descriptor array is NULL");
  if (L->n_seq <= 0) return fail(HC_ERR_ARG, "n_seq must be positive (got %d)", L->n_seq);
  if (L->D != 64 && L->D != 128) return fail(HC_ERR_UNSUPPORTED, "head_dim %d unsupported (64 or 128)", L->D);
  if (L->Hk <= 0 || L->Hq <= 0 || L->Hq % L->Hk)
    return fail(HC_ERR_ARG, "query heads %d must be a multiple of KV heads %d", L->Hq, L->Hk);
  const int G = L->Hq / L->Hk;
  if (G != 1 && G != 2 && G != 4 && G != 8) return fail(HC_ERR_UNSUPPORTED, "GQA group %d unsupported", G);
  if (L->dtype < HC_F32 || L->dtype > HC_BF16) return fail(HC_ERR_ARG, "bad dtype %d", L->dtype);
  if (L->F <= 0 || L->F > 4096) return fail(HC_ERR_ARG, "index dim %d out of range", L->F);
  if (L->max_r < 0 || L->max_r > 2048) return fail(HC_ERR_UNSUPPORTED, "lookahead %d above 2048", L->max_r);
  if (L->max_cap <= 0) return fail(HC_ERR_ARG, "max_cap must be positive");
  if (L->policy != HC_POLICY_HOTCOLD && L->policy != HC_POLICY_SNAPKV) return fail(HC_ERR_ARG, "bad policy");
  return HC_OK;
}

}  // namespace

namespace hc {
void set_last_error(const char* msg) { snprintf(g_err, sizeof(g_err), "%s", msg); }
}  // namespace hc

extern "C" {

const char* hc_version(void) { return "hotcold_b200 1.0 (sm_100a)"; }

int hc_host_device_pointer(const void* host, void** dev) {
  if (!host || !dev) return fail(HC_ERR_ARG, "NULL pointer argument");
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, host);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeHost) {
    (void)cudaGetLastError();
    return fail(HC_ERR_ARG, "not page-locked host memory registered with CUDA");
  }
  e = cudaHostGetDevicePointer(dev, const_cast<void*>(host), 0);
  return check_cuda(e, "host_device_pointer");
}
const char* hc_last_error(void) { return g_err; }

size_t hc_attention_dense_scratch_bytes(int B, int Hq, int Hk, int S, int D) {
  if (B <= 0 || Hk <= 0 || Hq <= 0 || S <= 0) return 0;
  const size_t part = hc::attention_part_bytes(B, Hq, Hk, D, S);
  const size_t ml = ((size_t)B * Hq * 2 * sizeof(float) + 255) & ~size_t(255);
  const size_t loss = ((size_t)B * S * sizeof(float) + 255) & ~size_t(255);
  return ((part + 255) & ~size_t(255)) + ml + loss;
}

int hc_attention_dense(const void* q, const void* k, const void* v, const uint8_t* mask, void* out,
                       int64_t* evict_idx, int B, int Hq, int Hk, int S, int D, int dtype, float scale,
                       int overflow_nan, int32_t* counters, void* scratch, size_t scratch_bytes, void* stream) {
  if (!q || !k || !v || !mask || !out || !counters) return fail(HC_ERR_ARG, "NULL tensor argument");
  if (B <= 0 || S <= 0) return fail(HC_ERR_ARG, "empty input (B=%d, S=%d)", B, S);
  if (D != 64 && D != 128) return fail(HC_ERR_UNSUPPORTED, "head_dim %d unsupported (64 or 128)", D);
  if (Hk <= 0 || Hq % Hk) return fail(HC_ERR_ARG, "Hq(%d)//N_REP must equal Hk(%d)", Hq, Hk);
  const int G = Hq / Hk;
  if (G != 1 && G != 2 && G != 4 && G != 8) return fail(HC_ERR_UNSUPPORTED, "GQA group %d unsupported", G);
  if (!aligned16(k) || !aligned16(v)) return fail(HC_ERR_ARG, "key/value must be 16-byte aligned");
  const size_t need = hc_attention_dense_scratch_bytes(B, Hq, Hk, S, D);
  if (!scratch || scratch_bytes < need) return fail(HC_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  char* base = reinterpret_cast<char*>(scratch);
  const size_t part = (hc::attention_part_bytes(B, Hq, Hk, D, S) + 255) & ~size_t(255);
  const size_t mlb = ((size_t)B * Hq * 2 * sizeof(float) + 255) & ~size_t(255);
  hc::AttnArgs a{};
  a.k = k;
  a.v = v;
  a.mask = mask;
  a.S = S;
  a.q = q;
  a.out = out;
  a.ml = evict_idx ? reinterpret_cast<float*>(base + part) : nullptr;
  a.part = reinterpret_cast<float*>(base);
  a.counters = counters;
  a.Hq = Hq;
  a.Hk = Hk;
  a.scale = scale;
  a.overflow_nan = overflow_nan;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = check_cuda(hc::launch_attention(a, dtype, D, G, B, S, true, st), "attention");
  if (rc || !evict_idx) return rc;
  return check_cuda(hc::launch_evict_idx(dtype, q, k, v, mask, a.ml, reinterpret_cast<float*>(base + part + mlb),
                                         evict_idx, B, Hq, Hk, S, D, scale, st),
                    "evict_idx");
}

int hc_append(const hc_layer* L, const void* q_pre, int64_t q_stride_seq, const void* k_pre, const void* v,
              int64_t kv_stride_seq, const void* cos, const void* sin, const int64_t* pos, void* q_post,
              void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!q_pre || !k_pre || !v || !pos || !q_post) return fail(HC_ERR_ARG, "NULL tensor argument");
  if ((cos == nullptr) != (sin == nullptr)) return fail(HC_ERR_ARG, "cos and sin must both be given or both NULL");
  if (!cos && !L->inv_freq) return fail(HC_ERR_ARG, "no cos/sin and no inv_freq");
  const int64_t esz = L->dtype == HC_F32 ? 4 : 2;
  if (!aligned16(q_pre) || !aligned16(k_pre) || !aligned16(v) || ((q_stride_seq * esz) & 15) ||
      ((kv_stride_seq * esz) & 15))
    return fail(HC_ERR_ARG, "query/key/value rows must be 16-byte aligned");
  return check_cuda(hc::launch_append(*L, q_pre, q_stride_seq, k_pre, v, kv_stride_seq, cos, sin, pos, q_post,
                                      reinterpret_cast<cudaStream_t>(stream)),
                    "append");
}

size_t hc_compress_scratch_bytes(const hc_layer* L, int S_max, int tq) {
  if (!L || S_max <= 0) return 0;
  return hc::compress_scratch_bytes(*L, S_max, tq);
}

int hc_compress_ex(const hc_layer* L, const void* q_obs, int64_t qs_seq, int64_t qs_head, int64_t qs_tok, int tq,
                   int S_dense, const void* src_k, const void* src_v, const void* src_kpre, int64_t ss_seq,
                   int64_t ss_head, int64_t ss_tok, const int64_t* src_pos, void* scratch, size_t scratch_bytes,
                   int n_evict_hint, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!q_obs || tq <= 0) return fail(HC_ERR_ARG, "no observation queries");
  const bool dense = src_k != nullptr;
  if (dense) {
    if (!src_v || !src_kpre || !src_pos) return fail(HC_ERR_ARG, "dense source needs k, v, k_pre and positions");
    if (S_dense <= 0) return fail(HC_ERR_ARG, "prompt length must be positive");
    if (!aligned16(src_k) || ((ss_tok * (L->dtype == HC_F32 ? 4 : 2)) & 15) || ((ss_head * (L->dtype == HC_F32 ? 4 : 2)) & 15) ||
        ((ss_seq * (L->dtype == HC_F32 ? 4 : 2)) & 15))
      return fail(HC_ERR_ARG, "post-RoPE key rows must be 16-byte aligned");
  }
  const int S_grid = dense ? S_dense : L->max_cap;
  const size_t need = hc::compress_scratch_bytes(*L, S_grid, tq);
  if (!scratch || scratch_bytes < need) return fail(HC_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  return check_cuda(hc::launch_compress(*L, q_obs, qs_seq, qs_head, qs_tok, tq, S_dense, src_k, src_v, src_kpre, ss_seq,
                                        ss_head, ss_tok, src_pos, scratch, n_evict_hint,
                                        reinterpret_cast<cudaStream_t>(stream)),
                    "compress");
}

int hc_compress(const hc_layer* L, const void* q_obs, int64_t qs_seq, int64_t qs_head, int64_t qs_tok, int tq,
                int S_dense, const void* src_k, const void* src_v, const void* src_kpre, int64_t ss_seq,
                int64_t ss_head, int64_t ss_tok, const int64_t* src_pos, void* scratch, size_t scratch_bytes,
                void* stream) {
  return hc_compress_ex(L, q_obs, qs_seq, qs_head, qs_tok, tq, S_dense, src_k, src_v, src_kpre, ss_seq, ss_head,
                        ss_tok, src_pos, scratch, scratch_bytes, 1 << 30, stream);
}

int hc_store_prompt(const hc_layer* L, int S, const void* src_k, const void* src_v, const void* src_kpre,
                    int64_t ss_seq, int64_t ss_head, int64_t ss_tok, const int64_t* src_pos, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!src_k || !src_v || !src_kpre || !src_pos) return fail(HC_ERR_ARG, "NULL tensor argument");
  if (S < 0 || S > L->max_cap) return fail(HC_ERR_ARG, "prompt of %d tokens does not fit %d slots", S, L->max_cap);
  return check_cuda(hc::launch_store_prompt(*L, S, src_k, src_v, src_kpre, ss_seq, ss_head, ss_tok, src_pos,
                                            reinterpret_cast<cudaStream_t>(stream)),
                    "store_prompt");
}

size_t hc_retrieve_scratch_bytes(const hc_layer* L) {
  if (!L) return 0;
  return hc::retrieve_scratch_bytes(*L);
}

int hc_retrieve_ex(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head, int64_t qd_tok, int P,
                   int n_pool, const float* extra_sum, int extra_n, const float* qvec_in, void* scratch,
                   size_t scratch_bytes, int max_count, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (L->max_r <= 0) return fail(HC_ERR_ARG, "lookahead_k is 0");
  if (L->max_ccap <= 0) return fail(HC_ERR_ARG, "no cold ring");
  if (q_dense && P <= 0) return fail(HC_ERR_ARG, "dense query needs P > 0");
  if (!qvec_in && !q_dense && n_pool <= 0 && extra_n <= 0) return fail(HC_ERR_ARG, "empty query pool");
  const size_t need = hc::retrieve_scratch_bytes(*L);
  if (!scratch || scratch_bytes < need) return fail(HC_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  if (max_count <= 0 || max_count > L->max_ccap) max_count = L->max_ccap;
  return check_cuda(hc::launch_retrieve(*L, q_dense, qd_seq, qd_head, qd_tok, P, n_pool, extra_sum, extra_n, qvec_in,
                                        scratch, max_count, reinterpret_cast<cudaStream_t>(stream)),
                    "retrieve");
}

int hc_retrieve_decode(const hc_layer* L, const void* q_pre, int64_t q_stride_seq, int n_pool, void* scratch,
                       size_t scratch_bytes, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!q_pre) return fail(HC_ERR_ARG, "NULL tensor argument");
  if (L->max_r <= 0) return fail(HC_ERR_ARG, "lookahead_k is 0");
  if (L->max_ccap <= 0) return fail(HC_ERR_ARG, "no cold ring");
  if (n_pool < 0) return fail(HC_ERR_ARG, "n_pool < 0");
  const size_t need = hc::retrieve_scratch_bytes(*L);
  if (!scratch || scratch_bytes < need) return fail(HC_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  const cudaError_t e = hc::launch_retrieve(*L, nullptr, 0, 0, 0, 0, n_pool, nullptr, 0, nullptr, scratch, L->max_ccap,
                                            reinterpret_cast<cudaStream_t>(stream), q_pre, q_stride_seq);
  if (e == cudaErrorNotSupported) {
    (void)cudaGetLastError();
    return fail(HC_ERR_UNSUPPORTED, "the fused retrieval kernel does not fit this layer");
  }
  return check_cuda(e, "retrieve_decode");
}

int hc_retrieve(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head, int64_t qd_tok, int P,
                int n_pool, const float* extra_sum, int extra_n, void* scratch, size_t scratch_bytes, void* stream) {
  return hc_retrieve_ex(L, q_dense, qd_seq, qd_head, qd_tok, P, n_pool, extra_sum, extra_n, nullptr, scratch,
                        scratch_bytes, 0, stream);
}

int hc_append_rotated(const hc_layer* L, const void* k_post, const void* k_pre, const void* v, int64_t kv_stride_seq,
                      const int64_t* pos, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!k_post || !k_pre || !v || !pos) return fail(HC_ERR_ARG, "NULL tensor argument");
  return check_cuda(hc::launch_append_rotated(*L, k_post, k_pre, v, kv_stride_seq, pos,
                                              reinterpret_cast<cudaStream_t>(stream)),
                    "append_rotated");
}

int hc_cold_append(const hc_layer* L, const void* k_pre, const void* v, int64_t s_seq, int64_t s_head, int64_t s_tok,
                   const int64_t* pos, const int64_t* evicted_idx, int Te, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!k_pre || !v || !pos || !evicted_idx) return fail(HC_ERR_ARG, "NULL tensor argument");
  if (Te < 0) return fail(HC_ERR_ARG, "negative token count");
  if (Te == 0) return HC_OK;
  if (L->max_ccap <= 0) return fail(HC_ERR_ARG, "no cold ring");
  return check_cuda(hc::launch_cold_append(*L, k_pre, v, s_seq, s_head, s_tok, pos, evicted_idx, Te,
                                           reinterpret_cast<cudaStream_t>(stream)),
                    "cold_append");
}

size_t hc_prompt_query_sum_scratch_bytes(const hc_layer* L) {
  return L ? hc::prompt_query_sum_scratch_bytes(*L) : 0;
}

int hc_prompt_query_sum(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head, int64_t qd_tok, int P,
                        float* out_sum, void* scratch, size_t scratch_bytes, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!q_dense || !out_sum || P <= 0) return fail(HC_ERR_ARG, "bad prompt query arguments");
  const size_t need = hc::prompt_query_sum_scratch_bytes(*L);
  if (!scratch || scratch_bytes < need) return fail(HC_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  return check_cuda(hc::launch_prompt_query_sum(*L, q_dense, qd_seq, qd_head, qd_tok, P, out_sum, scratch,
                                                reinterpret_cast<cudaStream_t>(stream)),
                    "prompt_query_sum");
}

size_t hc_attend_scratch_bytes(const hc_layer* L) {
  if (!L) return 0;
  return hc::attention_part_bytes(L->n_seq, L->Hq, L->Hk, L->D, L->max_r + L->max_cap);
}

int hc_attend(const hc_layer* L, const void* q_post, const int64_t* cur_pos, int use_held, void* out,
              int overflow_nan, void* scratch, size_t scratch_bytes, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!q_post || !cur_pos || !out || !L->counters) return fail(HC_ERR_ARG, "NULL tensor argument");
  const size_t need = hc_attend_scratch_bytes(L);
  if (!scratch || scratch_bytes < need) return fail(HC_ERR_SCRATCH, "scratch %zu < %zu bytes", scratch_bytes, need);
  hc::AttnArgs a{};
  a.desc = L->desc;
  a.cur_pos = cur_pos;
  a.use_held = use_held;
  a.q = q_post;
  a.out = out;
  a.part = reinterpret_cast<float*>(scratch);
  a.counters = L->counters;
  a.Hq = L->Hq;
  a.Hk = L->Hk;
  a.scale = L->scale;
  a.overflow_nan = overflow_nan;
  const int max_tokens = (use_held ? L->max_r : 0) + L->max_cap;
  return check_cuda(hc::launch_attention(a, L->dtype, L->D, L->Hq / L->Hk, L->n_seq, max_tokens, false,
                                         reinterpret_cast<cudaStream_t>(stream)),
                    "attend");
}

int hc_encode_kmap(void* out, const void* base, int dtype, int64_t rows, int D, int box_rows) {
  if (!out || !base) return fail(HC_ERR_ARG, "NULL argument");
  if (rows <= 0 || (D != 64 && D != 128) || box_rows < 1 || box_rows > 256)
    return fail(HC_ERR_ARG, "rows %lld, D %d, box_rows %d out of range", (long long)rows, D, box_rows);
  if (dtype != HC_F16 && dtype != HC_BF16) return fail(HC_ERR_UNSUPPORTED, "tensor maps serve 16-bit K only");
  if (reinterpret_cast<uintptr_t>(base) % 16) return fail(HC_ERR_ARG, "base must be 16-byte aligned");
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::mutex mu;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!encode) {
      cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
      void* fn = nullptr;
      const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        (void)cudaGetLastError();
        return fail(HC_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
      }
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  }
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1u, 1u};
  const CUresult r = encode(&m, dtype == HC_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  std::memcpy(out, &m, sizeof(m));
  return HC_OK;
}

static int step_checks(const hc_layer* L, int use_held) {
  if (!hc::step_parts(L->Hk)) return fail(HC_ERR_UNSUPPORTED, "KV heads %d do not divide a 16-CTA cluster", L->Hk);
  const size_t smem = hc::step_smem_bytes(*L, use_held);
  if (smem == 0 || smem > 227 * 1024)
    return fail(HC_ERR_UNSUPPORTED, "fused step needs %zu bytes of shared memory per CTA", smem);
  if (L->dtype != HC_F32 && !L->kmaps) return fail(HC_ERR_UNSUPPORTED, "16-bit fused step needs hc_layer.kmaps");
  return HC_OK;
}

int hc_step_check(const hc_layer* L, int use_held) {
  if (int rc = check_layer(L)) return rc;
  if (int rc = step_checks(L, use_held)) return rc;
  const cudaError_t e = hc::launch_step(*L, nullptr, 0, nullptr, nullptr, 0, nullptr, nullptr, nullptr, use_held, nullptr,
                                        0, 0, nullptr, true);
  if (e == cudaErrorNotSupported) {
    (void)cudaGetLastError();
    return fail(HC_ERR_UNSUPPORTED, "no resident 16-CTA cluster for this shared memory size");
  }
  return check_cuda(e, "step_check");
}

int hc_step(const hc_layer* L, const void* q_pre, int64_t q_stride_seq, const void* k_pre, const void* v,
            int64_t kv_stride_seq, const void* cos, const void* sin, const int64_t* pos, int use_held, void* out,
            int overflow_nan, int early, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!q_pre || !k_pre || !v || !pos || !out) return fail(HC_ERR_ARG, "NULL tensor argument");
  if ((cos == nullptr) != (sin == nullptr)) return fail(HC_ERR_ARG, "cos and sin must both be given or both NULL");
  if (!cos && !L->inv_freq) return fail(HC_ERR_ARG, "no cos/sin and no inv_freq");
  if (int rc = step_checks(L, use_held)) return rc;
  if (early & ~(HC_STEP_EARLY_HOT | HC_STEP_EARLY_HELD)) return fail(HC_ERR_ARG, "unknown early-read bits 0x%x", early);
  const cudaError_t e = hc::launch_step(*L, q_pre, q_stride_seq, k_pre, v, kv_stride_seq, cos, sin, pos, use_held, out,
                                        overflow_nan, early, reinterpret_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported) {
    (void)cudaGetLastError();
    return fail(HC_ERR_UNSUPPORTED, "no resident 16-CTA cluster for this shared memory size");
  }
  return check_cuda(e, "step");
}

int hc_shard_merge(const float* cand_score, const int32_t* cand_id, int n_shards, int k, int32_t* out_id,
                   float* out_score, void* stream) {
  if (!cand_score || !cand_id || !out_id) return fail(HC_ERR_ARG, "NULL tensor argument");
  if (n_shards <= 0 || k <= 0 || (long)n_shards * k > 4096)
    return fail(HC_ERR_UNSUPPORTED, "n_shards*k = %ld must be in 1..4096", (long)n_shards * k);
  return check_cuda(hc::launch_shard_merge(cand_score, cand_id, n_shards, k, out_id, out_score,
                                           reinterpret_cast<cudaStream_t>(stream)),
                    "shard_merge");
}

size_t hc_cold_topk_scratch_bytes(int64_t n_rows, int k) {
  return n_rows < 0 || k <= 0 ? 0 : hc::cold_topk_scratch_bytes(n_rows, k);
}

int hc_cold_topk(const float* index, int64_t n_rows, int F, int64_t id_base, const float* qvec, int k,
                 float* out_score, int32_t* out_id, void* scratch, size_t scratch_bytes, void* stream) {
  if (!qvec || !out_score || !out_id || !scratch || (n_rows > 0 && !index))
    return fail(HC_ERR_ARG, "NULL tensor argument");
  if (n_rows < 0 || F <= 0 || F > 4096 || k <= 0 || k > 256)
    return fail(HC_ERR_ARG, "n_rows %lld, F %d, k %d: need n_rows >= 0, 1 <= F <= 4096, 1 <= k <= 256",
                (long long)n_rows, F, k);
  if (id_base < 0 || id_base + n_rows > 0x7fffffffLL) return fail(HC_ERR_ARG, "ids must fit int32");
  if ((F & 3) == 0 && F <= 128 && (reinterpret_cast<uintptr_t>(index) & 15))
    return fail(HC_ERR_ARG, "index rows must be 16-byte aligned");
  if (scratch_bytes < hc::cold_topk_scratch_bytes(n_rows, k)) return fail(HC_ERR_ARG, "scratch too small");
  return check_cuda(hc::launch_cold_topk(index, n_rows, F, id_base, qvec, k, out_score, out_id, scratch,
                                         reinterpret_cast<cudaStream_t>(stream)),
                    "cold_topk");
}

int hc_retrieve_query(const hc_layer* L, const void* q_dense, int64_t qd_seq, int64_t qd_head, int64_t qd_tok, int P,
                      int n_pool, const float* extra_sum, int extra_n, float* out_qvec, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!out_qvec) return fail(HC_ERR_ARG, "NULL output");
  if (q_dense && P <= 0) return fail(HC_ERR_ARG, "P must be positive with q_dense");
  if (!q_dense && (n_pool < 0 || n_pool > 0x7fffffff)) return fail(HC_ERR_ARG, "bad n_pool");
  return check_cuda(hc::launch_retrieve_query(*L, q_dense, qd_seq, qd_head, qd_tok, P, n_pool, extra_sum, extra_n,
                                              out_qvec, reinterpret_cast<cudaStream_t>(stream)),
                    "retrieve_query");
}

int hc_splice_hits(const hc_layer* L, const int32_t* hit_ids, int k, void* stream) {
  if (int rc = check_layer(L)) return rc;
  if (!hit_ids || k < 0) return fail(HC_ERR_ARG, "NULL hit ids or negative k");
  return check_cuda(hc::launch_splice_hits(*L, hit_ids, k, reinterpret_cast<cudaStream_t>(stream)), "splice_hits");
}

}  // extern "C"
