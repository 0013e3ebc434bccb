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

#include <cooperative_groups.h>

#include "hc_topk.cuh"

namespace cg = cooperative_groups;

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
  const void* q_cur;     // optional: this step's pre-RoPE query (n_seq, Hq, D), the newest pool entry
  int64_t q_cur_ss;      // its stride between sequences (elements)
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
// Grid (max_r, n_seq), one CTA of kSpliceThreads per slot: the hit's D/2 cos/sin pairs once in
// shared memory, then 16-byte chunks of every head's key (with the rotate-half partner chunk)
// and value.
constexpr int kSpliceThreads = 128;

template <int DT, int D>
__global__ void __launch_bounds__(kSpliceThreads) splice_kernel(RetrieveArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int H = D / 2;
  constexpr int VEC = 16 / (int)sizeof(T);
  constexpr int CPR = D / VEC;  // 16-byte chunks per head row
  __shared__ float scs[2 * H];
  const hc_layer& L = a.L;
  const int j = blockIdx.x, s = blockIdx.y, tid = threadIdx.x;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  if (j >= d.r_max) return;
  const int phys = d.held_src[j];
  uint4* hk = reinterpret_cast<uint4*>(d.held_k);
  uint4* hv = reinterpret_cast<uint4*>(d.held_v);
  const int nq = L.Hk * CPR;
  if (phys < 0 || phys >= d.ccap) {
    for (int q = tid; q < nq; q += kSpliceThreads) {
      const int h = q / CPR, c = q % CPR;
      const size_t o = ((size_t)h * d.r_max + j) * CPR + c;
      hk[o] = make_uint4(0u, 0u, 0u, 0u);
      hv[o] = make_uint4(0u, 0u, 0u, 0u);
    }
    if (tid == 0) {
      d.held_pos[j] = 0;
      d.held_valid[j] = 0;
    }
    return;
  }
  const int64_t p = d.cold_pos[phys];
  for (int i = tid; i < H; i += kSpliceThreads) {
    float c, sn;
    rope_cs<DT>(L.inv_freq[i], p, L.rope_scaling, c, sn);
    scs[i] = c;
    scs[H + i] = sn;
  }
  __syncthreads();
  const uint4* ck = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(d.cold_kpre) + (size_t)phys * L.Hk * D);
  const uint4* cv = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(d.cold_v) + (size_t)phys * L.Hk * D);
  for (int q = tid; q < nq; q += kSpliceThreads) {
    const int h = q / CPR, c = q % CPR;
    const int cp = c < CPR / 2 ? c + CPR / 2 : c - CPR / 2;  // chunk of the rotate-half partner dims
    const uint4 xv = ck[(size_t)h * CPR + c], rv = ck[(size_t)h * CPR + cp], vv = cv[(size_t)h * CPR + c];
    const T* x = reinterpret_cast<const T*>(&xv);
    const T* r = reinterpret_cast<const T*>(&rv);
    uint4 ov;
    T* o = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int dd = c * VEC + e;
      const float rot = dd < H ? -E::to_f(r[e]) : E::to_f(r[e]);
      o[e] = E::from_f(rope_elem<DT>(E::to_f(x[e]), rot, scs[dd % H], scs[H + dd % H]));
    }
    const size_t off = ((size_t)h * d.r_max + j) * CPR + c;
    hk[off] = ov;
    hv[off] = vv;
  }
  if (tid == 0) {
    d.held_pos[j] = p;
    d.held_valid[j] = 1;
  }
}

// ------------------------------------------------------------------------------------------
// Fused retrieval: one 16-CTA cluster per sequence does the pooled query, the scan, the top-R
// and the splice. CTA r scans ring entries [r*count/16, (r+1)*count/16) (one lane per row),
// sorts them, sends its best R to CTA 0, which merges the candidates; every CTA then re-RoPEs a
// share of the (hit, head) pairs into the held segment.
// ------------------------------------------------------------------------------------------
constexpr int kRetThreads = 512;
constexpr int kRetWarps = kRetThreads / 32;
constexpr int kRetCluster = 16;

struct RetrSmem {
  size_t qv, red, keys, runs, cand, fin, sfin, qs, cs, total;
};
__host__ __device__ inline RetrSmem retr_smem(int F, int nloc2, int R2, int Hq = 0, int D = 0) {
  RetrSmem m{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t r = o; o += (b + 15) & ~size_t(15); return r; };
  m.qs = take((size_t)Hq * D * 4);  // the current query's rows, staged for the head mean
  m.qv = take((size_t)F * 4);
  m.red = take(32 * 4);
  m.keys = take((size_t)(nloc2 > 32 ? nloc2 : 32) * 8 + (R2 > 32 ? R2 : 32) * 8);
  {
    int nr = 1;
    while (nr * 32 < nloc2) nr <<= 1;
    m.runs = take((size_t)nr * (R2 > 32 ? R2 : 32) * 8);  // sorted 32-key runs as merge lists
  }
  m.cand = take((size_t)kRetCluster * (R2 > 32 ? R2 : 32) * 8);
  m.fin = take((size_t)R2 * 4);
  m.sfin = take((size_t)R2 * 4);
  m.cs = take((size_t)((R2 + kRetCluster - 1) / kRetCluster) * D * 4 + 16);  // cos/sin of this CTA's hits
  m.total = o;
  return m;
}

// Keys are unique 64-bit values (score key high, reversed index low), larger = better.
// Sort the 32 keys of a warp descending, one per lane (bitonic network over shuffles).
__device__ __forceinline__ unsigned long long warp_sort_desc_u64(unsigned long long x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, x, j);
      const bool desc = (lane & k) == 0;           // this 2k-block sorts descending
      const bool low = (lane & j) == 0;            // the lower lane of the pair
      const bool keep_max = (desc == low);
      x = keep_max ? (x > y ? x : y) : (x < y ? x : y);
    }
  return x;
}

// One warp merges two sorted-descending lists A and B of length R (a power of two, 32..256)
// into the R largest keys of both, sorted descending, written to `out` (may alias A). Lane l
// holds elements l + 32e: first the larger of A[i] and B[R-1-i] (a bitonic sequence holding
// the top R), then half-cleaners, inside a lane for strides >= 32 and across lanes below.
template <int E>
__device__ __forceinline__ void warp_merge_topr(const unsigned long long* A, const unsigned long long* B,
                                                unsigned long long* out) {
  constexpr int R = 32 * E;
  const int lane = threadIdx.x & 31;
  unsigned long long c[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane + 32 * e;
    const unsigned long long x = A[i], y = B[R - 1 - i];
    c[e] = x > y ? x : y;
  }
#pragma unroll
  for (int js = E / 2; js > 0; js >>= 1)  // stride 32*js: slots e and e + js of the same lane
#pragma unroll
    for (int e = 0; e < E; ++e)
      if ((e & js) == 0) {
        const unsigned long long x = c[e], y = c[e + js];
        c[e] = x > y ? x : y;
        c[e + js] = x > y ? y : x;
      }
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
    const bool low = (lane & j) == 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, c[e], j);
      c[e] = low ? (c[e] > y ? c[e] : y) : (c[e] < y ? c[e] : y);
    }
  }
  __syncwarp();
#pragma unroll
  for (int e = 0; e < E; ++e) out[lane + 32 * e] = c[e];
}

// Top-R of m sorted lists (m a power of two) stored at stride R in shared memory: a tree of
// warp merges, one barrier per level; the result is list 0. All threads of the block call.
template <int E>
__device__ __forceinline__ void block_merge_tree(unsigned long long* lists, int m) {
  constexpr int R = 32 * E;
  const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int step = 1; step < m; step <<= 1) {
    for (int q = warp; q < m / (2 * step); q += nw) {
      unsigned long long* A = lists + (size_t)(2 * q) * step * R;
      warp_merge_topr<E>(A, A + (size_t)step * R, A);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ void block_merge_tree_any(unsigned long long* lists, int m, int RL) {
  switch (RL) {
    case 32: block_merge_tree<1>(lists, m); break;
    case 64: block_merge_tree<2>(lists, m); break;
    case 128: block_merge_tree<4>(lists, m); break;
    default: block_merge_tree<8>(lists, m); break;
  }
}

__device__ __forceinline__ void block_merge_topr_any(unsigned long long* lists, int m, int RL) {
  switch (RL) {
    case 32: block_merge_tree<1>(lists, m); break;
    case 64: block_merge_tree<2>(lists, m); break;
    case 128: block_merge_tree<4>(lists, m); break;
    default: block_merge_tree<8>(lists, m); break;
  }
}

template <int DT, int D>
__global__ void __launch_bounds__(kRetThreads, 1) retr_kernel(RetrieveArgs a, int nloc2, int R2) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int H = D / 2;
  cg::cluster_group cluster = cg::this_cluster();
  const hc_layer& L = a.L;
  const int rank = (int)cluster.block_rank(), s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  extern __shared__ __align__(16) unsigned char smem[];
  const RetrSmem M = retr_smem(L.F, nloc2, R2, L.Hq, D);
  float* qv = reinterpret_cast<float*>(smem + M.qv);
  float* qs = reinterpret_cast<float*>(smem + M.qs);
  float* red = reinterpret_cast<float*>(smem + M.red);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem + M.keys);
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem + M.cand);
  unsigned long long* runs = reinterpret_cast<unsigned long long*>(smem + M.runs);
  int* fin = reinterpret_cast<int*>(smem + M.fin);
  int* sfin = reinterpret_cast<int*>(smem + M.sfin);
  cluster_arrive_relaxed();  // started; waited on before the first remote store

  const hc_seq_desc d = L.desc[s];
  pdl_wait();
  hc_seq_state* st = d.st;
  const int count = max(0, min(st->cold_count, d.ccap)), head = st->cold_head;
  const int R = d.r_max, k = min(R, count), F = L.F;

  // ---- pooled query vector (controller.py:184-188,243-248), rounded like the reference ----
  // this step's query rows in one round trip, summed over heads in head order below
  if (a.q_cur && !a.qvec_in) {
    const T* q = reinterpret_cast<const T*>(a.q_cur) + (size_t)s * a.q_cur_ss;
    constexpr int kQ = 16;
    float tq[kQ];
#pragma unroll
    for (int j = 0; j < kQ; ++j)
      if (tid + j * kRetThreads < L.Hq * D) tq[j] = E::to_f(q[tid + j * kRetThreads]);
#pragma unroll
    for (int j = 0; j < kQ; ++j)
      if (tid + j * kRetThreads < L.Hq * D) qs[tid + j * kRetThreads] = tq[j];
    for (int k2 = tid + kQ * kRetThreads; k2 < L.Hq * D; k2 += kRetThreads) qs[k2] = E::to_f(q[k2]);
    __syncthreads();
  }
  if (a.qvec_in) {
    for (int f = tid; f < F; f += kRetThreads) qv[f] = a.qvec_in[(size_t)s * F + f];
  } else {
    float m2 = 0.f, ss = 0.f;
    if (tid < D) {
      float tot = 0.f;
      int npos = 0;
      if (a.q_cur) {  // the newest entry: this step's query, as the query-pool push rounds it
        float acc = 0.f;
        for (int hh = 0; hh < L.Hq; ++hh) acc += qs[hh * D + tid];
        tot += E::to_f(E::from_f(acc / (float)L.Hq));
        npos = 1;
      }
      if (a.q_dense) {
        const T* q = reinterpret_cast<const T*>(a.q_dense) + (size_t)s * a.qd_seq;
        for (int pp = 0; pp < a.P; ++pp) {
          float acc = 0.f;
#pragma unroll 8
          for (int hh = 0; hh < L.Hq; ++hh) acc += E::to_f(q[(size_t)hh * a.qd_head + (size_t)pp * a.qd_tok + tid]);
          tot += E::round(acc / (float)L.Hq);
        }
        npos += a.P;
      } else {
        const T* qw = reinterpret_cast<const T*>(d.qwin);
        const int qh = st->qwin_head;
        // newest first; loads batched, the sum in that order
        constexpr int kW = 8;
        for (int i0 = 1; i0 <= a.n_pool && d.p_max > 0; i0 += kW) {
          float wv[kW];
#pragma unroll
          for (int j = 0; j < kW; ++j) {
            const int i = i0 + j;
            wv[j] = i <= a.n_pool ? E::to_f(qw[(size_t)(((qh - i) % d.p_max + d.p_max) % d.p_max) * D + tid]) : 0.f;
          }
#pragma unroll
          for (int j = 0; j < kW; ++j)
            if (i0 + j <= a.n_pool) tot += wv[j];
        }
        npos += a.n_pool;
        if (a.extra_sum && a.extra_n > 0) {
          tot += a.extra_sum[(size_t)s * D + tid];
          npos += a.extra_n;
        }
      }
      m2 = E::round(tot / (float)max(npos, 1));  // mean over positions, model dtype
      const float x = tid < F ? m2 : 0.f;
      ss = x * x;
    }
    ss = warp_sum(ss);
    if (lane == 0 && warp < D / 32) red[warp] = ss;
    __syncthreads();
    if (tid < D) {
      float tot2 = 0.f;
      for (int w = 0; w < D / 32; ++w) tot2 += red[w];
      if (tid < F) {
        if (L.normalize) {
          const float n = E::round(sqrtf(tot2));
          const float den = fmaxf(n, E::round(1e-12f));
          qv[tid] = E::round(m2 / den);
        } else {
          qv[tid] = m2;
        }
      }
    }
    for (int f = D + tid; f < F; f += kRetThreads) qv[f] = 0.f;
  }
  __syncthreads();
  if (rank == 0 && a.qvec)
    for (int f = tid; f < F; f += kRetThreads) a.qvec[(size_t)s * F + f] = qv[f];

  // ---- scan this CTA's share of the ring in age order ---------------------------------------
  // 8 lanes per row (coalesced 128-byte reads). Lane l keeps the four-element partials of
  // chunks l, l+8, l+16, l+24 and sums them, then across lanes, in the order of a 32-lane
  // xor-reduction, so each score equals the warp-per-row scan's.
  const int l0 = rank * count / kRetCluster, l1 = (rank + 1) * count / kRetCluster, nloc = l1 - l0;
  // the sorted runs: warp w's 32-key runs occupy keys[w*32 ...]; runs are merged as lists of R2
  const int nruns = (nloc + 31) >> 5;
  if ((F & 3) == 0 && F <= 128) {
    const int nv = F >> 2, sub = lane & 7, rg = lane >> 3;
    float4 qc[4];
#pragma unroll
    for (int m = 0; m < 4; ++m)
      qc[m] = sub + 8 * m < nv ? reinterpret_cast<const float4*>(qv)[sub + 8 * m] : make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int U = 2;  // row groups per iteration, loads of both in flight
    for (int base = warp * 4; base < nloc; base += 4 * kRetWarps * U) {
      float4 x[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * 4 * kRetWarps + rg;
        int phys = head + l0 + i;
        if (phys >= d.ccap) phys -= d.ccap;
        const float4* row = reinterpret_cast<const float4*>(d.cold_vec + (size_t)phys * F);
#pragma unroll
        for (int m = 0; m < 4; ++m)
          x[u][m] = (i < nloc && sub + 8 * m < nv) ? row[sub + 8 * m] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * 4 * kRetWarps + rg;
        float pt[4];
#pragma unroll
        for (int m = 0; m < 4; ++m)
          pt[m] = x[u][m].x * qc[m].x + x[u][m].y * qc[m].y + x[u][m].z * qc[m].z + x[u][m].w * qc[m].w;
        float v = (pt[0] + pt[2]) + (pt[1] + pt[3]);  // levels 16 and 8 of the xor tree
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        if (sub == 0 && i < nloc) keys[i] = ((unsigned long long)fkey(v) << 32) | (0xffffffffu - (uint32_t)(l0 + i));
      }
    }
  } else {
    for (int i = warp; i < nloc; i += kRetWarps) {
      const int l = l0 + i;
      int phys = head + l;
      if (phys >= d.ccap) phys -= d.ccap;
      float acc = 0.f;
      for (int f = lane; f < F; f += 32) acc = fmaf(d.cold_vec[(size_t)phys * F + f], qv[f], acc);
      acc = warp_sum(acc);
      if (lane == 0) keys[i] = ((unsigned long long)fkey(acc) << 32) | (0xffffffffu - (uint32_t)l);
    }
  }
  __syncthreads();
  // runs of 32 sorted by their warps, padded to R2 when R2 > 32, then merged to the best R2
  {
    const int RL = R2 > 32 ? R2 : 32;  // list length of the merges
    for (int r = warp; r < nruns; r += kRetWarps) {
      const int i = r * 32 + lane;
      unsigned long long x = i < nloc ? keys[i] : 0ull;
      x = warp_sort_desc_u64(x);
      __syncwarp();
      runs[(size_t)r * RL + lane] = x;
      for (int j = 32 + lane; j < RL; j += 32) runs[(size_t)r * RL + j] = 0ull;
    }
    int m = 1;
    while (m < nruns) m <<= 1;
    for (int i = nruns * RL + tid; i < m * RL; i += kRetThreads) runs[i] = 0ull;
    __syncthreads();
    block_merge_topr_any(runs, m, RL);
    for (int j = tid; j < RL; j += kRetThreads) keys[j] = nruns > 0 ? runs[j] : 0ull;
    __syncthreads();
  }

  // ---- best R of every CTA to CTA 0, which merges them --------------------------------------------
  const int RL = R2 > 32 ? R2 : 32;
  cluster_wait();
  {
    unsigned long long* dst = cluster.map_shared_rank(cand, 0) + (size_t)rank * RL;
    const int nk = min(R, nloc);
    for (int j = tid; j < RL; j += kRetThreads) dst[j] = j < nk ? keys[j] : 0ull;
  }
  cluster.sync();
  if (rank == 0) {
    block_merge_topr_any(cand, kRetCluster, RL);
    // hits in score order, ties to the older entry (controller.py:274-293)
    for (int j = tid; j < R; j += kRetThreads) {
      int phys = -1;
      if (j < k) {
        const long l = (long)(0xffffffffu - (uint32_t)(cand[j] & 0xffffffffu));
        phys = (int)(((long)head + l) % d.ccap);
      }
      fin[j] = phys;
      d.held_src[j] = phys;
    }
    if (tid == 0) {
      if (a.hits) a.hits[s] = k;
      st->n_hits = k;
      st->held_len = R;
    }
  }
  cluster.sync();
  for (int j = tid; j < R; j += kRetThreads) sfin[j] = cluster.map_shared_rank(fin, 0)[j];
  __syncthreads();
  cluster_arrive_relaxed();  // done reading CTA 0's shared memory

  // ---- splice (patch.py:94-102 with HF's LlamaRotaryEmbedding and apply_rotary_pos_emb in
  //      the model dtype): CTA r takes hits j = r, r+16, ...; each hit's cos/sin once, then a
  //      warp per (hit, head); slots past the hits are zero and invalid (controller.py:259-262)
  T* hk = reinterpret_cast<T*>(d.held_k);
  T* hv = reinterpret_cast<T*>(d.held_v);
  float* scs = reinterpret_cast<float*>(smem + M.cs);  // [local hit][H] cos, then [local hit][H] sin
  const int nmine = R > rank ? (R - rank + kRetCluster - 1) / kRetCluster : 0;
  for (int t = tid; t < nmine * H; t += kRetThreads) {
    const int jl = t / H, i = t - jl * H, j = rank + jl * kRetCluster;
    const int phys = sfin[j];
    float c = 0.f, sn = 0.f;
    if (phys >= 0 && phys < d.ccap) rope_cs<DT>(L.inv_freq[i], d.cold_pos[phys], L.rope_scaling, c, sn);
    scs[jl * D + i] = c;
    scs[jl * D + H + i] = sn;
  }
  __syncthreads();
  for (int q = warp; q < nmine * L.Hk; q += kRetWarps) {
    const int jl = q / L.Hk, hh = q - jl * L.Hk, j = rank + jl * kRetCluster;
    const int phys = sfin[j];
    const size_t doff = ((size_t)hh * d.r_max + j) * D;
    if (phys < 0 || phys >= d.ccap) {
      for (int dd = lane; dd < D; dd += 32) {
        hk[doff + dd] = E::from_f(0.f);
        hv[doff + dd] = E::from_f(0.f);
      }
      if (hh == 0 && lane == 0) {
        d.held_pos[j] = 0;
        d.held_valid[j] = 0;
      }
      continue;
    }
    const T* ck = reinterpret_cast<const T*>(d.cold_kpre) + ((size_t)phys * L.Hk + hh) * D;
    const T* cv = reinterpret_cast<const T*>(d.cold_v) + ((size_t)phys * L.Hk + hh) * D;
    float kx[D / 32], kr[D / 32];
    T vx[D / 32];
#pragma unroll
    for (int u = 0; u < D / 32; ++u) {
      const int dd = lane + 32 * u;
      kx[u] = E::to_f(ck[dd]);
      kr[u] = dd < H ? -E::to_f(ck[dd + H]) : E::to_f(ck[dd - H]);
      vx[u] = cv[dd];
    }
#pragma unroll
    for (int u = 0; u < D / 32; ++u) {
      const int dd = lane + 32 * u;
      const float c = scs[jl * D + (dd % H)], sn = scs[jl * D + H + (dd % H)];
      hk[doff + dd] = E::from_f(rope_elem<DT>(kx[u], kr[u], c, sn));
      hv[doff + dd] = vx[u];
    }
    if (hh == 0 && lane == 0) {
      d.held_pos[j] = d.cold_pos[phys];
      d.held_valid[j] = 1;
    }
  }
  cluster_wait();
}

// ------------------------------------------------------------------------------------------
// Exact inner-product top-k over a block of index rows: the search of IndexFlatIP
// (controller.py:274) over one token-range shard of the cold index. Rows are scored with the
// arithmetic of the ring scan above (8 lanes per row, the same xor-tree order), so a row's
// score does not depend on which shard holds it and the union of the shards' top-k holds the
// exact global top-k. Ids are id_base + row; ties go to the lower id.
//   topk_scan_kernel   CTA c scans rows [c*per_cta, (c+1)*per_cta) in batches of 1024: keys
//                      into shared memory, warp-sorted 32-key runs, a merge tree to the best
//                      RL, merged into the CTA's running best; writes its list of RL keys;
//   topk_merge_kernel  CTA b merges lists [32b, 32b+32); the last CTA to finish (an atomic
//                      ticket, no waiting) merges those results and writes the top k.
// ------------------------------------------------------------------------------------------
constexpr int kTopkThreads = 512;
constexpr int kTopkBatch = 1024;
constexpr int kTopkFanIn = 32;

struct TopkArgs {
  const float* index;
  int64_t n;
  int F;
  int64_t id_base;
  const float* q;
  int k, RL, per_cta, nA, nB;
  unsigned long long* lists;   // [nA][RL]
  unsigned long long* lists2;  // [nB][RL]
  unsigned int* ticket;
  float* out_score;
  int32_t* out_id;
};

__host__ __device__ inline size_t topk_scan_smem(int F, int RL) {
  return (size_t)((F + 3) & ~3) * 4 + (size_t)kTopkBatch * 8 + (size_t)(kTopkBatch / 32) * RL * 8 + (size_t)RL * 8;
}

__device__ __forceinline__ void warp_merge_topr_any(const unsigned long long* A, const unsigned long long* B,
                                                    unsigned long long* out, int RL) {
  switch (RL) {
    case 32: warp_merge_topr<1>(A, B, out); break;
    case 64: warp_merge_topr<2>(A, B, out); break;
    case 128: warp_merge_topr<4>(A, B, out); break;
    default: warp_merge_topr<8>(A, B, out); break;
  }
}

__global__ void __launch_bounds__(kTopkThreads) topk_scan_kernel(TopkArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int F = a.F, RL = a.RL;
  float* qv = reinterpret_cast<float*>(smem);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem + (size_t)((F + 3) & ~3) * 4);
  unsigned long long* runs = keys + kTopkBatch;
  unsigned long long* best = runs + (size_t)(kTopkBatch / 32) * RL;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = kTopkThreads / 32;
  pdl_wait();
  for (int f = tid; f < F; f += kTopkThreads) qv[f] = a.q[f];
  for (int j = tid; j < RL; j += kTopkThreads) best[j] = 0ull;
  __syncthreads();
  const int64_t r0 = (int64_t)blockIdx.x * a.per_cta;
  const int64_t r1 = min(a.n, r0 + a.per_cta);
  const bool vec = (F & 3) == 0 && F <= 128;
  const int nv = F >> 2, sub = lane & 7, rg = lane >> 3;
  float4 qc[4];
  if (vec) {
#pragma unroll
    for (int m = 0; m < 4; ++m)
      qc[m] = sub + 8 * m < nv ? reinterpret_cast<const float4*>(qv)[sub + 8 * m] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int64_t b0 = r0; b0 < r1; b0 += kTopkBatch) {
    const int nb = (int)min((int64_t)kTopkBatch, r1 - b0);
    if (vec) {
      constexpr int U = 2;
      for (int base = warp * 4; base < nb; base += 4 * NW * U) {
        float4 x[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * 4 * NW + rg;
          const float4* row = reinterpret_cast<const float4*>(a.index + (size_t)(b0 + i) * F);
#pragma unroll
          for (int m = 0; m < 4; ++m)
            x[u][m] = (i < nb && sub + 8 * m < nv) ? row[sub + 8 * m] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * 4 * NW + rg;
          float pt[4];
#pragma unroll
          for (int m = 0; m < 4; ++m)
            pt[m] = x[u][m].x * qc[m].x + x[u][m].y * qc[m].y + x[u][m].z * qc[m].z + x[u][m].w * qc[m].w;
          float v = (pt[0] + pt[2]) + (pt[1] + pt[3]);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 2);
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          if (sub == 0 && i < nb)
            keys[i] = ((unsigned long long)fkey(v) << 32) | (0xffffffffu - (uint32_t)(a.id_base + b0 + i));
        }
      }
    } else {
      for (int i = warp; i < nb; i += NW) {
        const float* row = a.index + (size_t)(b0 + i) * F;
        float acc = 0.f;
        for (int f = lane; f < F; f += 32) acc = fmaf(row[f], qv[f], acc);
        acc = warp_sum(acc);
        if (lane == 0) keys[i] = ((unsigned long long)fkey(acc) << 32) | (0xffffffffu - (uint32_t)(a.id_base + b0 + i));
      }
    }
    __syncthreads();
    const int nruns = (nb + 31) >> 5;
    for (int r = warp; r < nruns; r += NW) {
      const int i = r * 32 + lane;
      unsigned long long x = i < nb ? keys[i] : 0ull;
      x = warp_sort_desc_u64(x);
      __syncwarp();
      runs[(size_t)r * RL + lane] = x;
      for (int j = 32 + lane; j < RL; j += 32) runs[(size_t)r * RL + j] = 0ull;
    }
    int m = 1;
    while (m < nruns) m <<= 1;
    for (int i = nruns * RL + tid; i < m * RL; i += kTopkThreads) runs[i] = 0ull;
    __syncthreads();
    block_merge_topr_any(runs, m, RL);
    if (warp == 0) warp_merge_topr_any(best, runs, best, RL);
    __syncthreads();
  }
  unsigned long long* dst = a.lists + (size_t)blockIdx.x * RL;
  for (int j = tid; j < RL; j += kTopkThreads) dst[j] = best[j];
}

__global__ void __launch_bounds__(kTopkThreads) topk_merge_kernel(TopkArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  unsigned long long* sl = reinterpret_cast<unsigned long long*>(smem);
  __shared__ int last;
  const int RL = a.RL, tid = threadIdx.x, b = blockIdx.x;
  pdl_wait();
  for (int i = tid; i < kTopkFanIn * RL; i += kTopkThreads) {
    const int l = b * kTopkFanIn + i / RL;
    sl[i] = l < a.nA ? a.lists[(size_t)l * RL + i % RL] : 0ull;
  }
  __syncthreads();
  block_merge_tree_any(sl, kTopkFanIn, RL);
  for (int j = tid; j < RL; j += kTopkThreads) a.lists2[(size_t)b * RL + j] = sl[j];
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(a.ticket, 1u) == (unsigned)(a.nB - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  int m = 1;
  while (m < a.nB) m <<= 1;
  for (int i = tid; i < m * RL; i += kTopkThreads)
    sl[i] = i / RL < a.nB ? __ldcg(a.lists2 + i) : 0ull;
  __syncthreads();
  block_merge_tree_any(sl, m, RL);
  for (int j = tid; j < a.k; j += kTopkThreads) {
    const unsigned long long key = sl[j];
    const bool live = key != 0ull;
    const uint32_t u = (uint32_t)(key >> 32);
    const uint32_t bits = (u & 0x80000000u) ? (u & 0x7fffffffu) : ~u;
    a.out_score[j] = live ? __uint_as_float(bits) : kNegInf;
    a.out_id[j] = live ? (int32_t)(0xffffffffu - (uint32_t)(key & 0xffffffffu)) : -1;
  }
  if (tid == 0) *a.ticket = 0u;  // ready for the next call
}

// Held slots from given hits: hit_ids (n_seq, k) are live cold entries in age order (0 = the
// oldest), -1 for none; slot j takes hit j (the gather order of controller.py:277-285).
__global__ void hits_kernel(hc_layer L, const int32_t* hit_ids, int k) {
  const int s = blockIdx.x;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const int count = max(0, min(d.st->cold_count, d.ccap)), head = d.st->cold_head;
  __shared__ int nh;
  if (threadIdx.x == 0) nh = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < d.r_max; j += blockDim.x) {
    const int id = j < k ? hit_ids[(size_t)s * k + j] : -1;
    const bool ok = id >= 0 && id < count;
    if (id >= count) set_status(d.st, HC_DEV_INDEX);
    d.held_src[j] = ok ? (int)(((long)head + id) % d.ccap) : -1;
    if (ok) atomicAdd(&nh, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    d.st->n_hits = nh;
    d.st->held_len = d.r_max;
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

static int pow2_at_least(int x) {
  int n = 1;
  while (n < x) n <<= 1;
  return n;
}

// The fused cluster kernel, or cudaErrorNotSupported when its shared memory or cluster does not fit.
template <int DT, int D>
static cudaError_t retr_cluster_t(const RetrieveArgs& a, cudaStream_t stream) {
  const hc_layer& L = a.L;
  const int nloc2 = pow2_at_least(max(32, (L.max_ccap + kRetCluster - 1) / kRetCluster));
  const int R2 = pow2_at_least(max(1, L.max_r));
  const size_t smem = retr_smem(L.F, nloc2, R2, L.Hq, D).total;
  if (smem > 200 * 1024 || L.F > 4096 || R2 > 256) return cudaErrorNotSupported;
  auto kern = retr_kernel<DT, D>;
  static std::mutex mu;
  static int ok_dev[64] = {0};  // 0 unknown, 1 schedulable, -1 not
  static size_t ok_smem[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kRetCluster, L.n_seq);
  cfg.blockDim = dim3(kRetThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kRetCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  {
    std::lock_guard<std::mutex> lock(mu);
    const int di = dev & 63;
    if (ok_dev[di] == 0 || ok_smem[di] < smem) {
      e = ensure_smem(kern, smem);
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      int clusters = 0;
      e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
      if (e != cudaSuccess) return e;
      ok_dev[di] = clusters >= 1 ? 1 : -1;
      ok_smem[di] = smem;
    }
    if (ok_dev[di] < 0) return cudaErrorNotSupported;
  }
  return cudaLaunchKernelEx(&cfg, kern, a, nloc2, R2);
}

template <int DT, int D>
static cudaError_t retrieve_t(RetrieveArgs a, int max_count, cudaStream_t stream) {
  const hc_layer& L = a.L;
  cudaError_t e = retr_cluster_t<DT, D>(a, stream);
  if (e != cudaErrorNotSupported) return e;
  (void)cudaGetLastError();
  if (a.q_cur) return cudaErrorNotSupported;  // the four-kernel path takes no separate current query
  e = cudaSuccess;
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
  return launch_pdl(splice_kernel<DT, D>, dim3(max(L.max_r, 1), L.n_seq), dim3(kSpliceThreads), 0, stream, a);
}

cudaError_t launch_retrieve(const hc_layer& L, const void* qd, int64_t q0, int64_t q1, int64_t q2, int P, int n_pool,
                            const float* extra_sum, int extra_n, const float* qvec_in, void* scratch, int max_count,
                            cudaStream_t stream, const void* q_cur, int64_t q_cur_ss) {
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
  a.q_cur = q_cur;
  a.q_cur_ss = q_cur_ss;
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

static int topk_rl(int k) {
  int RL = 32;
  while (RL < k) RL <<= 1;
  return RL;
}
static int topk_ctas(int64_t n) {
  int64_t c = (n + 255) / 256;
  if (c > 296) c = 296;
  return c < 1 ? 1 : (int)c;
}
size_t cold_topk_scratch_bytes(int64_t n, int k) {
  const int RL = topk_rl(k), nA = topk_ctas(n), nB = (nA + kTopkFanIn - 1) / kTopkFanIn;
  return al256((size_t)nA * RL * 8) + al256((size_t)nB * RL * 8) + 256;
}

cudaError_t launch_cold_topk(const float* index, int64_t n, int F, int64_t id_base, const float* q, int k,
                             float* out_score, int32_t* out_id, void* scratch, cudaStream_t stream) {
  TopkArgs a{};
  a.index = index;
  a.n = n;
  a.F = F;
  a.id_base = id_base;
  a.q = q;
  a.k = k;
  a.RL = topk_rl(k);
  a.nA = topk_ctas(n);
  a.per_cta = (int)((n + a.nA - 1) / a.nA);
  a.nB = (a.nA + kTopkFanIn - 1) / kTopkFanIn;
  char* base = reinterpret_cast<char*>(scratch);
  a.lists = reinterpret_cast<unsigned long long*>(base);
  a.lists2 = reinterpret_cast<unsigned long long*>(base + al256((size_t)a.nA * a.RL * 8));
  a.ticket = reinterpret_cast<unsigned int*>(base + al256((size_t)a.nA * a.RL * 8) + al256((size_t)a.nB * a.RL * 8));
  a.out_score = out_score;
  a.out_id = out_id;
  cudaError_t e = cudaMemsetAsync(a.ticket, 0, sizeof(unsigned int), stream);
  if (e != cudaSuccess) return e;
  const size_t s1 = topk_scan_smem(F, a.RL), s2 = (size_t)kTopkFanIn * a.RL * 8;
  e = ensure_smem(topk_scan_kernel, s1);
  if (e == cudaSuccess) e = ensure_smem(topk_merge_kernel, s2);
  if (e == cudaSuccess) e = launch_pdl(topk_scan_kernel, dim3(a.nA), dim3(kTopkThreads), s1, stream, a);
  if (e == cudaSuccess) e = launch_pdl(topk_merge_kernel, dim3(a.nB), dim3(kTopkThreads), s2, stream, a);
  return e;
}

template <int DT, int D>
static cudaError_t splice_hits_t(RetrieveArgs a, const int32_t* hit_ids, int k, cudaStream_t stream) {
  const hc_layer& L = a.L;
  cudaError_t e = launch_pdl(hits_kernel, dim3(L.n_seq), dim3(256), 0, stream, L, hit_ids, k);
  if (e != cudaSuccess) return e;
  return launch_pdl(splice_kernel<DT, D>, dim3(max(L.max_r, 1), L.n_seq), dim3(kSpliceThreads), 0, stream, a);
}

template <int DT, int D>
static cudaError_t query_t(RetrieveArgs a, cudaStream_t stream) {
  return launch_pdl(query_kernel<DT, D>, dim3(a.L.n_seq), dim3(D), 0, stream, a);
}

cudaError_t launch_retrieve_query(const hc_layer& L, const void* qd, int64_t q0, int64_t q1, int64_t q2, int P,
                                  int n_pool, const float* extra_sum, int extra_n, float* qvec, cudaStream_t stream) {
  RetrieveArgs a{};
  a.L = L;
  a.q_dense = qd;
  a.qd_seq = q0; a.qd_head = q1; a.qd_tok = q2;
  a.P = P;
  a.n_pool = n_pool;
  a.extra_sum = extra_sum;
  a.extra_n = extra_n;
  a.qvec = qvec;
  HC_DISPATCH_DT_D(L.dtype, L.D, query_t, a, stream);
}

cudaError_t launch_splice_hits(const hc_layer& L, const int32_t* hit_ids, int k, cudaStream_t stream) {
  RetrieveArgs a{};
  a.L = L;
  HC_DISPATCH_DT_D(L.dtype, L.D, splice_hits_t, a, hit_ids, k, stream);
}

}  // namespace hc
