// Internal launcher interface shared by the kernel files and the C ABI layer.
#pragma once
#include "hc_common.cuh"

namespace hc {

// A compression of S hot tokens: keep the top n_top of the first `prefix` plus the tail;
// `nobs` caps the observation query rows; active = 0 when nothing is compressed.
struct Plan {
  int S, prefix, ntop, nobs, active;
};

struct AttnArgs {
  // slab mode
  const hc_seq_desc* desc;
  const int64_t* cur_pos;
  int use_held;
  // dense mode
  const void* k;
  const void* v;
  const uint8_t* mask;
  int S;
  // common
  const void* q;      // (n_seq, Hq, D)
  void* out;          // (n_seq, Hq, D)
  float* ml;          // optional (n_seq, Hq, 2): final max and sum per head (dense mode)
  float* part;        // scratch partials
  int32_t* counters;  // (n_seq*Hk)
  int Hq, Hk, max_chunks;
  float scale;
  int overflow_nan;
};

cudaError_t launch_attention(const AttnArgs& a, int dtype, int D, int G, int n_seq, int max_tokens, bool dense,
                             cudaStream_t stream);
size_t attention_part_bytes(int n_seq, int Hq, int Hk, int D, int max_tokens);
cudaError_t launch_evict_idx(int dtype, const void* q, const void* k, const void* v, const uint8_t* mask,
                             const float* ml, float* loss, int64_t* out, int B, int Hq, int Hk, int S, int D,
                             float scale, cudaStream_t stream);
cudaError_t launch_append(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                          const void* c, const void* sn, const int64_t* pos, void* qo, cudaStream_t st);
cudaError_t launch_store_prompt(const hc_layer& L, int S, const void* a, const void* b, const void* c, int64_t s0,
                                int64_t s1, int64_t s2, const int64_t* pos, cudaStream_t st);
cudaError_t launch_prompt_query_sum(const hc_layer& L, const void* q, int64_t a, int64_t b, int64_t c, int P,
                                    float* out, void* scratch, cudaStream_t st);
size_t prompt_query_sum_scratch_bytes(const hc_layer& L);
cudaError_t launch_compress(const hc_layer& L, const void* q_obs, int64_t qs0, int64_t qs1, int64_t qs2, int tq,
                            int S_dense, const void* sk, const void* sv, const void* skp, int64_t ss0, int64_t ss1,
                            int64_t ss2, const int64_t* spos, void* scratch, int n_evict_hint, cudaStream_t stream);
size_t compress_scratch_bytes(const hc_layer& L, int S_max, int tq);
cudaError_t launch_retrieve(const hc_layer& L, const void* qd, int64_t q0, int64_t q1, int64_t q2, int P, int n_pool,
                            const float* extra_sum, int extra_n, const float* qvec_in, void* scratch, int max_count,
                            cudaStream_t stream, const void* q_cur = nullptr, int64_t q_cur_ss = 0);
cudaError_t launch_append_rotated(const hc_layer& L, const void* kpost, const void* kpre, const void* v, int64_t kvss,
                                  const int64_t* pos, cudaStream_t st);
cudaError_t launch_cold_append(const hc_layer& L, const void* kpre, const void* v, int64_t s0, int64_t s1, int64_t s2,
                               const int64_t* pos, const int64_t* idx, int Te, cudaStream_t st);
size_t retrieve_scratch_bytes(const hc_layer& L);
cudaError_t launch_step(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                        const void* c, const void* sn, const int64_t* pos, int use_held, void* out, int overflow_nan,
                        int early, cudaStream_t stream, bool check_only = false);
size_t step_smem_bytes(const hc_layer& L, int use_held);
int step_parts(int Hk);

// Set the message hc_last_error() returns on the calling thread.
void set_last_error(const char* msg);

size_t cold_topk_scratch_bytes(int64_t n, int k);
cudaError_t launch_cold_topk(const float* index, int64_t n, int F, int64_t id_base, const float* q, int k,
                             float* out_score, int32_t* out_id, void* scratch, cudaStream_t stream);
cudaError_t launch_retrieve_query(const hc_layer& L, const void* qd, int64_t q0, int64_t q1, int64_t q2, int P,
                                  int n_pool, const float* extra_sum, int extra_n, float* qvec, cudaStream_t stream);
cudaError_t launch_splice_hits(const hc_layer& L, const int32_t* hit_ids, int k, cudaStream_t stream);
cudaError_t launch_shard_merge(const float* cs, const int32_t* cid, int n_shards, int k, int32_t* out_id,
                               float* out_score, cudaStream_t stream);

}  // namespace hc
