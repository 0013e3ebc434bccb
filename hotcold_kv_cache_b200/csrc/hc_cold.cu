// Cold-store retrieval in HBM.
//
// The reference keeps the cold tier in host memory and searches it with a CPU FAISS
// IndexFlatIP on a daemon thread (controller.py:250-293), then copies the hits to the GPU
// on a side stream (controller.py:344-380) and re-rotates them on the next poll
// (patch.py:94-102,249). Here the index vectors and payload live in an HBM ring and one
// decode step runs four kernels on the caller's stream:
//   query_kernel   pooled query vector (controller.py:184-188,243-248), rounded to the
//                  model dtype at the same steps as the reference's torch ops;
//   scan_kernel    exact inner products of every live ring row with the query, written in
//                  ring (age) order — a memory-bound GEMV;
//   pick_kernel    exact top-R (ties to the older entry), sorted by score;
//   splice_kernel  gather of the hits, RoPE at their original positions, write into the
//                  held segment; unused slots are zeroed and marked invalid.

#include "hc_topk.cuh"

namespace hc {

struct RetrieveArgs {
  hc_layer L;
  const void* q_dense;
  int64_t qd_seq, qd_head, qd_tok;
  int P;             // dense: positions; pool: entries to average
  int n_pool;        // pool mode: newest entries of the query ring
  const float* extra_sum;
  int extra_n;
  const float* qvec_in;  // optional given query vectors [n_seq][F]
  float* qvec;       // [n_seq][F]
  float* scores;     // [n_seq][max_ccap]
  uint8_t* sel;      // [n_seq][max_ccap]
  int* hits;         // [n_seq]
};

// One CTA (D threads) per sequence.
template <int DT, int D>
__global__ void query_kernel(RetrieveArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  const hc_layer& L = a.L;
  const int s = blockIdx.x, dd = threadIdx.x;
  __shared__ float red[32];
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  float tot = 0.f;
  int npos = 0;
  if (a.q_dense) {
    const T* q = reinterpret_cast<const T*>(a.q_dense) + (size_t)s * a.qd_seq;
    for (int p = 0; p < a.P; ++p) {
      float acc = 0.f;
      for (int h = 0; h < L.Hq; ++h) acc += E::to_f(q[(size_t)h * a.qd_head + (size_t)p * a.qd_tok + dd]);
      tot += E::round(acc / (float)L.Hq);  // mean over heads in the model dtype
    }
    npos = a.P;
  } else {
    const T* qw = reinterpret_cast<const T*>(d.qwin);
    const int head = d.st->qwin_head;
    for (int i = 1; i <= a.n_pool; ++i) {
      const int slot = ((head - i) % d.p_max + d.p_max) % d.p_max;
      tot += E::to_f(qw[(size_t)slot * D + dd]);
    }
    npos = a.n_pool;
    if (a.extra_sum && a.extra_n > 0) {
      tot += a.extra_sum[(size_t)s * D + dd];
      npos += a.extra_n;
    }
  }
  const float m2 = E::round(tot / (float)max(npos, 1));  // mean over positions, model dtype
  // pad/crop to F (controller.py:166-171), F.normalize in the model dtype
  const float x = dd < L.F ? m2 : 0.f;
  float ss = x * x;
  ss = warp_sum(ss);
  if ((dd & 31) == 0) red[dd >> 5] = ss;
  __syncthreads();
  float tot2 = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot2 += red[w];
  float* out = a.qvec + (size_t)s * L.F;
  if (L.normalize) {
    const float n = E::round(sqrtf(tot2));
    const float eps = E::round(1e-12f);
    const float den = fmaxf(n, eps);
    if (dd < L.F) out[dd] = E::round(m2 / den);
  } else if (dd < L.F) {
    out[dd] = m2;
  }
  for (int f = D + dd; f < L.F; f += blockDim.x) out[f] = 0.f;
}

// scores[s][l] = cold_vec[(head + l) % ccap] . q for live ring entries l < count.
// A warp per row, 16-byte loads.
__global__ void __launch_bounds__(256) scan_kernel(RetrieveArgs a) {
  const hc_layer& L = a.L;
  const int s = blockIdx.y;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const int count = max(0, min(d.st->cold_count, d.ccap)), head = d.st->cold_head;
  const int lane = threadIdx.x & 31;
  const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  const float* q = (a.qvec_in ? a.qvec_in : a.qvec) + (size_t)s * L.F;
  float* sc = a.scores + (size_t)s * L.max_ccap;
  if ((L.F & 3) == 0 && L.F <= 128) {
    const int nv = L.F >> 2;
    const float4 qv = lane < nv ? reinterpret_cast<const float4*>(q)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int l = w0; l < count; l += nw) {
      const int phys = (int)(((long)head + l) % d.ccap);
      float acc = 0.f;
      if (lane < nv) {
        const float4 x = reinterpret_cast<const float4*>(d.cold_vec + (size_t)phys * L.F)[lane];
        acc = x.x * qv.x + x.y * qv.y + x.z * qv.z + x.w * qv.w;
      }
      acc = warp_sum(acc);
      if (lane == 0) sc[l] = acc;
    }
  } else {
    for (int l = w0; l < count; l += nw) {
      const int phys = (int)(((long)head + l) % d.ccap);
      float acc = 0.f;
      for (int f = lane; f < L.F; f += 32) acc = fmaf(d.cold_vec[(size_t)phys * L.F + f], q[f], acc);
      acc = warp_sum(acc);
      if (lane == 0) sc[l] = acc;
    }
  }
}

// Top-R of the scanned scores (ties to the lower ring index = the older entry), sorted by
// score descending. One CTA of 1024 threads per sequence.
__global__ void __launch_bounds__(1024) pick_kernel(RetrieveArgs a) {
  const hc_layer& L = a.L;
  const int s = blockIdx.x, tid = threadIdx.x;
  __shared__ int sh[kTopkSmemInts];
  __shared__ uint32_t skey[2048];
  __shared__ int32_t sid[2048];
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const int count = max(0, min(d.st->cold_count, d.ccap)), head = d.st->cold_head;
  const int R = d.r_max;
  const int k = min(R, count);
  float* sc = a.scores + (size_t)s * L.max_ccap;
  uint8_t* sel = a.sel + (size_t)s * L.max_ccap;
  if (k > 0) block_topk_flags([&](int i) { return sc[i]; }, count, k, sel, sh);
  // gather the k selected (key, index) pairs in index order
  int base_out = 0;
  for (int base = 0; base < count; base += blockDim.x) {
    const int i = base + tid;
    const int f = (i < count && k > 0) ? sel[i] : 0;
    int tot;
    const int r = block_exclusive_scan(f, sh + 256, tot);
    if (f && base_out + r < 2048) {
      skey[base_out + r] = fkey(sc[i]);
      sid[base_out + r] = i;
    }
    base_out += tot;
  }
  int n2 = 1;
  while (n2 < k) n2 <<= 1;
  for (int i = k + tid; i < n2; i += blockDim.x) {
    skey[i] = 0u;
    sid[i] = 0x7fffffff;
  }
  __syncthreads();
  if (k > 1) block_sort_desc(skey, sid, n2);
  for (int j = tid; j < R; j += blockDim.x) d.held_src[j] = j < k ? (int)(((long)head + sid[j]) % d.ccap) : -1;
  if (tid == 0) {
    a.hits[s] = k;
    d.st->n_hits = k;
    d.st->held_len = R;
  }
}

// Held slot j <- hit j: RoPE of the pre-RoPE key at its position (patch.py:94-102 with HF's
// LlamaRotaryEmbedding and apply_rotary_pos_emb, rounded in the model dtype), value, position,
// valid flag; slots past the hits are zero and invalid (controller.py:259-262).
// Grid (ceil(max_r/8), n_seq), a warp per slot.
template <int DT, int D>
__global__ void __launch_bounds__(256) splice_kernel(RetrieveArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int H = D / 2;
  const hc_layer& L = a.L;
  const int s = blockIdx.y;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const int j = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (j >= d.r_max) return;
  const int phys = d.held_src[j];
  T* hk = reinterpret_cast<T*>(d.held_k);
  T* hv = reinterpret_cast<T*>(d.held_v);
  if (phys < 0 || phys >= d.ccap) {
    for (int h = 0; h < L.Hk; ++h)
      for (int dd = lane; dd < D; dd += 32) {
        hk[((size_t)h * d.r_max + j) * D + dd] = E::from_f(0.f);
        hv[((size_t)h * d.r_max + j) * D + dd] = E::from_f(0.f);
      }
    if (lane == 0) {
      d.held_pos[j] = 0;
      d.held_valid[j] = 0;
    }
    return;
  }
  const int64_t p = d.cold_pos[phys];
  const T* ck = reinterpret_cast<const T*>(d.cold_kpre) + (size_t)phys * L.Hk * D;
  const T* cv = reinterpret_cast<const T*>(d.cold_v) + (size_t)phys * L.Hk * D;
  for (int dd = lane; dd < D; dd += 32) {
    float c, sn;
    rope_cs<DT>(L.inv_freq[dd % H], p, L.rope_scaling, c, sn);
    for (int h = 0; h < L.Hk; ++h) {
      const float x = E::to_f(ck[(size_t)h * D + dd]);
      const float r = dd < H ? -E::to_f(ck[(size_t)h * D + dd + H]) : E::to_f(ck[(size_t)h * D + dd - H]);
      hk[((size_t)h * d.r_max + j) * D + dd] = E::from_f(rope_elem<DT>(x, r, c, sn));
      hv[((size_t)h * d.r_max + j) * D + dd] = cv[(size_t)h * D + dd];
    }
  }
  if (lane == 0) {
    d.held_pos[j] = p;
    d.held_valid[j] = 1;
  }
}

// ------------------------------------------------------------------------------------------
// multi-GPU: merge per-shard candidates into the global top-k (ties to the lower id)
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) shard_merge_kernel(const float* cs, const int32_t* cid, int n, int k,
                                                           int32_t* out_id, float* out_score) {
  __shared__ uint32_t key[4096];
  __shared__ int32_t id[4096];
  int n2 = 1;
  while (n2 < n) n2 <<= 1;
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    const bool live = i < n && cid[i] >= 0;
    key[i] = live ? fkey(cs[i]) : 0u;
    id[i] = live ? cid[i] : 0x7fffffff;
  }
  __syncthreads();
  block_sort_desc(key, id, n2);
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const bool live = j < n2 && id[j] != 0x7fffffff;
    out_id[j] = live ? id[j] : -1;
    if (out_score) {
      const uint32_t u = key[j];
      const uint32_t b = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
      out_score[j] = live ? __uint_as_float(b) : kNegInf;
    }
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
struct RetrieveLayout {
  size_t qvec, scores, sel, hits, total;
};
static size_t al256(size_t x) { return (x + 255) & ~size_t(255); }
RetrieveLayout retrieve_layout(const hc_layer& L) {
  RetrieveLayout r{};
  size_t off = 0;
  auto take = [&](size_t b) { size_t o = off; off += al256(b); return o; };
  r.qvec = take((size_t)L.n_seq * L.F * sizeof(float));
  r.scores = take((size_t)L.n_seq * L.max_ccap * sizeof(float));
  r.sel = take((size_t)L.n_seq * L.max_ccap);
  r.hits = take((size_t)L.n_seq * sizeof(int));
  r.total = off;
  return r;
}
size_t retrieve_scratch_bytes(const hc_layer& L) { return retrieve_layout(L).total; }

template <int DT, int D>
static cudaError_t retrieve_t(RetrieveArgs a, int max_count, cudaStream_t stream) {
  const hc_layer& L = a.L;
  cudaError_t e = cudaSuccess;
  if (!a.qvec_in) {
    e = launch_pdl(query_kernel<DT, D>, dim3(L.n_seq), dim3(D), 0, stream, a);
    if (e != cudaSuccess) return e;
  }
  int blocks = (max_count + 7) / 8;
  if (blocks > 592) blocks = 592;
  if (blocks < 1) blocks = 1;
  e = launch_pdl(scan_kernel, dim3(blocks, L.n_seq), dim3(256), 0, stream, a);
  if (e != cudaSuccess) return e;
  e = launch_pdl(pick_kernel, dim3(L.n_seq), dim3(1024), 0, stream, a);
  if (e != cudaSuccess) return e;
  return launch_pdl(splice_kernel<DT, D>, dim3((L.max_r + 7) / 8, L.n_seq), dim3(256), 0, stream, a);
}

cudaError_t launch_retrieve(const hc_layer& L, const void* qd, int64_t q0, int64_t q1, int64_t q2, int P, int n_pool,
                            const float* extra_sum, int extra_n, const float* qvec_in, void* scratch, int max_count,
                            cudaStream_t stream) {
  const RetrieveLayout lay = retrieve_layout(L);
  char* base = reinterpret_cast<char*>(scratch);
  RetrieveArgs a{};
  a.L = L;
  a.q_dense = qd;
  a.qd_seq = q0; a.qd_head = q1; a.qd_tok = q2;
  a.P = P;
  a.n_pool = n_pool;
  a.extra_sum = extra_sum;
  a.extra_n = extra_n;
  a.qvec_in = qvec_in;
  a.qvec = reinterpret_cast<float*>(base + lay.qvec);
  a.scores = reinterpret_cast<float*>(base + lay.scores);
  a.sel = reinterpret_cast<uint8_t*>(base + lay.sel);
  a.hits = reinterpret_cast<int*>(base + lay.hits);
  HC_DISPATCH_DT_D(L.dtype, L.D, retrieve_t, a, max_count, stream);
}

cudaError_t launch_shard_merge(const float* cs, const int32_t* cid, int n_shards, int k, int32_t* out_id,
                               float* out_score, cudaStream_t stream) {
  shard_merge_kernel<<<1, 1024, 0, stream>>>(cs, cid, n_shards * k, k, out_id, out_score);
  return cudaGetLastError();
}

}  // namespace hc
