// Hot-tier updates: the decode-step append and the prompt store.
//
// The reference appends with four torch.cat calls per decode step (cache.py:145-148),
// copying the whole hot cache every step. Here the hot slab is preallocated with
// budget + 1 physical slots; a new token takes a slot from the free-slot stack and
// its logical position is recorded in hot_ord, so an append writes one token.

#include <cooperative_groups.h>

#include "hc_common.cuh"

namespace cg = cooperative_groups;

namespace hc {

// One CTA per sequence. Rotates the new query and key (patch.py:161-162 with HF's
// apply_rotary_pos_emb), appends (k_post, v, k_pre, pos) to the slab, and pushes the
// mean over query heads of the pre-RoPE query into the query pool ring
// (controller.py:240-241; the pool is later averaged by controller.py:185).
// 16 bytes of elements as floats, and back.
template <int DT>
__device__ __forceinline__ void load_vec(const typename Elem<DT>::T* __restrict__ p, float* f) {
  unpack16<DT>(*reinterpret_cast<const uint4*>(p), f);
}
template <int DT>
__device__ __forceinline__ void store_vec(typename Elem<DT>::T* __restrict__ p, const float* f) {
  using T = typename Elem<DT>::T;
  constexpr int V = 16 / sizeof(T);
  alignas(16) T tmp[V];
#pragma unroll
  for (int e = 0; e < V; ++e) tmp[e] = Elem<DT>::from_f(f[e]);
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(tmp);
}

// RoPE of one (head, 16-byte chunk) pair: lo = x[j*V..], hi = x[H + j*V..].
template <int DT, int D>
__device__ __forceinline__ void rope_pair(const typename Elem<DT>::T* __restrict__ x, int j, const float* c,
                                          const float* s, float* lo, float* hi) {
  constexpr int H = D / 2, V = 16 / sizeof(typename Elem<DT>::T);
  float xl[V], xh[V];
  load_vec<DT>(x + j * V, xl);
  load_vec<DT>(x + H + j * V, xh);
#pragma unroll
  for (int e = 0; e < V; ++e) {
    lo[e] = rope_elem<DT>(xl[e], -xh[e], c[e], s[e]);
    hi[e] = rope_elem<DT>(xh[e], xl[e], c[V + e], s[V + e]);
  }
}

template <int DT, int D>
__global__ void __launch_bounds__(256) append_kernel(hc_layer L, const void* __restrict__ q_pre_, int64_t qss,
                                                     const void* __restrict__ k_pre_, const void* __restrict__ v_,
                                                     int64_t kvss, const void* __restrict__ cos_,
                                                     const void* __restrict__ sin_, const int64_t* __restrict__ pos,
                                                     void* __restrict__ q_post_) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int H = D / 2;
  constexpr int V = 16 / sizeof(T);
  constexpr int NV = H / V;  // 16-byte chunks per half row
  const int s = blockIdx.x;
  __shared__ float sc[D], ss[D];
  __shared__ int sSlot, sOrdAt;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  hc_seq_state* st = d.st;
  const int64_t p = pos[s];
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    if (cos_) {
      sc[i] = E::load(reinterpret_cast<const T*>(cos_) + (size_t)s * D + i);
      ss[i] = E::load(reinterpret_cast<const T*>(sin_) + (size_t)s * D + i);
    } else {
      float c, sn;
      rope_cs<DT>(L.inv_freq[i % H], p, L.rope_scaling, c, sn);
      sc[i] = c;
      ss[i] = sn;
    }
  }
  if (threadIdx.x == 0) {
    const int nf = st->n_free, nh = st->n_hot;
    int slot = -1;
    if (nf > 0 && nh < d.cap) {
      slot = d.hot_free[nf - 1];
      if (slot < 0 || slot >= d.cap) {
        set_status(st, HC_DEV_INDEX);
        slot = -1;
      }
    } else {
      set_status(st, HC_DEV_CAPACITY);
    }
    sSlot = slot;
    sOrdAt = nh;
  }
  __syncthreads();
  const int slot = sSlot;
  const T* __restrict__ q = reinterpret_cast<const T*>(q_pre_) + (size_t)s * qss;
  const T* __restrict__ k = reinterpret_cast<const T*>(k_pre_) + (size_t)s * kvss;
  const T* __restrict__ v = reinterpret_cast<const T*>(v_) + (size_t)s * kvss;
  T* __restrict__ qo = reinterpret_cast<T*>(q_post_) + (size_t)s * L.Hq * D;
  // one work item = (head, 16-byte chunk j of the first half) -> both RoPE halves
  const int n_q = L.Hq * NV, n_k = L.Hk * NV;
  for (int it = threadIdx.x; it < n_q + n_k; it += blockDim.x) {
    const bool isq = it < n_q;
    const int h = (isq ? it : it - n_q) / NV, j = (isq ? it : it - n_q) % NV;
    float c[2 * V], sn[2 * V], lo[V], hi[V];
#pragma unroll
    for (int e = 0; e < V; ++e) {
      c[e] = sc[j * V + e];
      sn[e] = ss[j * V + e];
      c[V + e] = sc[H + j * V + e];
      sn[V + e] = ss[H + j * V + e];
    }
    if (isq) {
      rope_pair<DT, D>(q + (size_t)h * D, j, c, sn, lo, hi);
      store_vec<DT>(qo + (size_t)h * D + j * V, lo);
      store_vec<DT>(qo + (size_t)h * D + H + j * V, hi);
    } else if (slot >= 0) {
      // post-RoPE key, pre-RoPE key and value of KV head h into the slab
      rope_pair<DT, D>(k + (size_t)h * D, j, c, sn, lo, hi);
      const size_t off = ((size_t)h * d.cap + slot) * D;
      T* hk = reinterpret_cast<T*>(d.hot_k) + off;
      T* hp = reinterpret_cast<T*>(d.hot_kpre) + off;
      T* hv = reinterpret_cast<T*>(d.hot_v) + off;
      store_vec<DT>(hk + j * V, lo);
      store_vec<DT>(hk + H + j * V, hi);
      *reinterpret_cast<uint4*>(hp + j * V) = *reinterpret_cast<const uint4*>(k + (size_t)h * D + j * V);
      *reinterpret_cast<uint4*>(hp + H + j * V) = *reinterpret_cast<const uint4*>(k + (size_t)h * D + H + j * V);
      *reinterpret_cast<uint4*>(hv + j * V) = *reinterpret_cast<const uint4*>(v + (size_t)h * D + j * V);
      *reinterpret_cast<uint4*>(hv + H + j * V) = *reinterpret_cast<const uint4*>(v + (size_t)h * D + H + j * V);
    }
  }
  // query pool: mean over heads of the pre-RoPE query, rounded to the model dtype
  if (d.p_max > 0) {
    const int qh = ((st->qwin_head % d.p_max) + d.p_max) % d.p_max;
    T* qw = reinterpret_cast<T*>(d.qwin) + (size_t)qh * D;
    for (int dd = threadIdx.x; dd < D; dd += blockDim.x) {
      float acc = 0.f;
#pragma unroll 8
      for (int h = 0; h < L.Hq; ++h) acc += E::to_f(q[(size_t)h * D + dd]);
      qw[dd] = E::from_f(acc / (float)L.Hq);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (slot >= 0) {
      d.hot_ord[sOrdAt] = slot;
      d.hot_pos[slot] = p;
      st->n_hot = sOrdAt + 1;
      st->n_free = st->n_free - 1;
    }
    if (d.p_max > 0) st->qwin_head = (((st->qwin_head % d.p_max) + d.p_max) % d.p_max + 1) % d.p_max;
  }
  pdl_launch_dependents();
}

// Append of already-rotated keys (HotColdLayer.update on a one-token step, cache.py:145-148).
template <int DT, int D>
__global__ void __launch_bounds__(256) append_rotated_kernel(hc_layer L, const void* kpost_, const void* kpre_,
                                                             const void* v_, int64_t kvss, const int64_t* pos) {
  using T = typename Elem<DT>::T;
  const int s = blockIdx.x;
  __shared__ int sSlot, sOrdAt;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  hc_seq_state* st = d.st;
  if (threadIdx.x == 0) {
    const int nf = st->n_free, nh = st->n_hot;
    int slot = -1;
    if (nf > 0 && nh < d.cap) slot = d.hot_free[nf - 1];
    if (slot < 0 || slot >= d.cap) {
      set_status(st, HC_DEV_CAPACITY);
      slot = -1;
    }
    sSlot = slot;
    sOrdAt = nh;
  }
  __syncthreads();
  const int slot = sSlot;
  if (slot < 0) return;
  const T* kq = reinterpret_cast<const T*>(kpost_) + (size_t)s * kvss;
  const T* kp = reinterpret_cast<const T*>(kpre_) + (size_t)s * kvss;
  const T* vv = reinterpret_cast<const T*>(v_) + (size_t)s * kvss;
  for (int i = threadIdx.x; i < L.Hk * D; i += blockDim.x) {
    const int h = i / D, dd = i % D;
    const size_t off = ((size_t)h * d.cap + slot) * D + dd;
    reinterpret_cast<T*>(d.hot_k)[off] = kq[i];
    reinterpret_cast<T*>(d.hot_kpre)[off] = kp[i];
    reinterpret_cast<T*>(d.hot_v)[off] = vv[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    d.hot_ord[sOrdAt] = slot;
    d.hot_pos[slot] = pos[s];
    st->n_hot = sOrdAt + 1;
    st->n_free = st->n_free - 1;
  }
}

// Prompt store without compression: token t -> physical slot t, logical order = identity.
template <int DT, int D>
__global__ void store_prompt_kernel(hc_layer L, int S, const void* sk, const void* sv, const void* skp, int64_t ss_seq,
                                    int64_t ss_head, int64_t ss_tok, const int64_t* spos) {
  using T = typename Elem<DT>::T;
  const int s = blockIdx.y;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const int S_src = S;  // row stride of the position array
  S = min(S, d.cap);
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int t = warp; t < S; t += nw) {
    for (int h = 0; h < L.Hk; ++h) {
      const size_t src = (size_t)s * ss_seq + (size_t)h * ss_head + (size_t)t * ss_tok;
      const size_t dst = ((size_t)h * d.cap + t) * D;
      for (int dd = lane; dd < D; dd += 32) {
        reinterpret_cast<T*>(d.hot_k)[dst + dd] = reinterpret_cast<const T*>(sk)[src + dd];
        reinterpret_cast<T*>(d.hot_v)[dst + dd] = reinterpret_cast<const T*>(sv)[src + dd];
        reinterpret_cast<T*>(d.hot_kpre)[dst + dd] = reinterpret_cast<const T*>(skp)[src + dd];
      }
    }
    if (lane == 0) {
      d.hot_pos[t] = spos[(size_t)s * S_src + t];
      d.hot_ord[t] = t;
    }
  }
  if (blockIdx.x == 0) {
    // free stack holds the unused slots, the lowest on top
    for (int i = threadIdx.x; i < d.cap - S; i += blockDim.x) d.hot_free[i] = d.cap - 1 - i;
    if (threadIdx.x == 0) {
      d.st->n_hot = S;
      d.st->n_free = d.cap - S;
    }
  }
}

// Sum over prompt positions of the head-mean pre-RoPE query (each mean rounded to the model
// dtype, as torch's mean over heads returns that dtype), fp32 (n_seq, D), in two passes over the
// whole GPU. Pass 1: CTA b of a sequence takes the contiguous positions [b P / nb, (b+1) P / nb);
// a lane holds 16 bytes of a row (VE elements) and sums them over the heads in head order, rounds
// the mean and adds it over its positions; the CTA reduces its lanes in a fixed order into
// part[s][b][D]. Pass 2 adds the nb partials of a sequence in block order. Deterministic.
constexpr int kPqsThreads = 256;
constexpr int kPqsBlocks = 296;  // CTAs per sequence at most (two waves of 148 SMs)

size_t prompt_query_sum_scratch_bytes(const hc_layer& L) {
  return (size_t)L.n_seq * kPqsBlocks * L.D * sizeof(float);
}

template <int DT, int D, bool VEC>
__global__ void __launch_bounds__(kPqsThreads) pqs_part_kernel(hc_layer L, const void* q_, int64_t qs, int64_t qh,
                                                                int64_t qt, int P, float* part) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VE = 16 / sizeof(T);  // elements per 16-byte chunk
  constexpr int CPR = D / VE;         // chunks per row
  constexpr int PPW = 32 / CPR;       // positions per warp pass
  constexpr int NW = kPqsThreads / 32;
  static_assert(CPR <= 32 && 32 % CPR == 0, "a row must fit one warp");
  __shared__ float red[NW * PPW][D];
  const int s = blockIdx.y, b = blockIdx.x, nb = gridDim.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = lane % CPR, sub = lane / CPR;
  const int p0 = (int)((long)b * P / nb), p1 = (int)((long)(b + 1) * P / nb);
  pdl_wait();
  const T* q = reinterpret_cast<const T*>(q_) + (size_t)s * qs + (size_t)c * VE;
  float tot[VE];
#pragma unroll
  for (int e = 0; e < VE; ++e) tot[e] = 0.f;
  for (int p = p0 + warp * PPW + sub; p < p1; p += NW * PPW) {
    const T* row = q + (size_t)p * qt;
    float acc[VE];
#pragma unroll
    for (int e = 0; e < VE; ++e) acc[e] = 0.f;
    int h = 0;
    // heads in groups of 8: the loads of a group are in flight together, the sum keeps the head order
    for (; h + 8 <= L.Hq; h += 8) {
      float x[8][VE];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if constexpr (VEC) {
          unpack16<DT>(*reinterpret_cast<const uint4*>(row + (size_t)(h + u) * qh), x[u]);
        } else {
#pragma unroll
          for (int e = 0; e < VE; ++e) x[u][e] = E::to_f(row[(size_t)(h + u) * qh + e]);
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int e = 0; e < VE; ++e) acc[e] += x[u][e];
    }
    for (; h < L.Hq; ++h)
#pragma unroll
      for (int e = 0; e < VE; ++e) acc[e] += E::to_f(row[(size_t)h * qh + e]);
#pragma unroll
    for (int e = 0; e < VE; ++e) tot[e] += E::round(acc[e] / (float)L.Hq);
  }
#pragma unroll
  for (int e = 0; e < VE; ++e) red[warp * PPW + sub][c * VE + e] = tot[e];
  __syncthreads();
  for (int dd = threadIdx.x; dd < D; dd += kPqsThreads) {
    float t = 0.f;
    for (int j = 0; j < NW * PPW; ++j) t += red[j][dd];
    part[((size_t)s * nb + b) * D + dd] = t;
  }
}

template <int D>
__global__ void pqs_sum_kernel(const float* part, int nb, float* out) {
  const int s = blockIdx.x;
  pdl_wait();
  for (int dd = threadIdx.x; dd < D; dd += blockDim.x) {
    float t = 0.f;
    for (int b = 0; b < nb; ++b) t += part[((size_t)s * nb + b) * D + dd];
    out[(size_t)s * D + dd] = t;
  }
}

template <int DT, int D>
static cudaError_t append_t(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                            const void* c, const void* sn, const int64_t* pos, void* qo, cudaStream_t st) {
  return launch_pdl(append_kernel<DT, D>, dim3(L.n_seq), dim3(256), 0, st, L, q, qss, k, v, kvss, c, sn, pos, qo);
}
cudaError_t launch_append(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                          const void* c, const void* sn, const int64_t* pos, void* qo, cudaStream_t st) {
  HC_DISPATCH_DT_D(L.dtype, L.D, append_t, L, q, qss, k, v, kvss, c, sn, pos, qo, st);
}

template <int DT, int D>
static cudaError_t append_rot_t(const hc_layer& L, const void* kq, const void* kp, const void* v, int64_t kvss,
                                const int64_t* pos, cudaStream_t st) {
  return launch_pdl(append_rotated_kernel<DT, D>, dim3(L.n_seq), dim3(256), 0, st, L, kq, kp, v, kvss, pos);
}
cudaError_t launch_append_rotated(const hc_layer& L, const void* kq, const void* kp, const void* v, int64_t kvss,
                                  const int64_t* pos, cudaStream_t st) {
  HC_DISPATCH_DT_D(L.dtype, L.D, append_rot_t, L, kq, kp, v, kvss, pos, st);
}

template <int DT, int D>
static cudaError_t store_t(const hc_layer& L, int S, const void* a, const void* b, const void* c, int64_t s0,
                           int64_t s1, int64_t s2, const int64_t* pos, cudaStream_t st) {
  const int blocks = (S + 7) / 8 < 148 ? (S + 7) / 8 : 148;
  return launch_pdl(store_prompt_kernel<DT, D>, dim3(blocks > 0 ? blocks : 1, L.n_seq), dim3(256), 0, st, L, S, a, b,
                    c, s0, s1, s2, pos);
}
cudaError_t launch_store_prompt(const hc_layer& L, int S, const void* a, const void* b, const void* c, int64_t s0,
                                int64_t s1, int64_t s2, const int64_t* pos, cudaStream_t st) {
  HC_DISPATCH_DT_D(L.dtype, L.D, store_t, L, S, a, b, c, s0, s1, s2, pos, st);
}

template <int DT, int D>
static cudaError_t pqs_t(const hc_layer& L, const void* q, int64_t a, int64_t b, int64_t c, int P, float* out,
                         float* part, cudaStream_t st) {
  using T = typename Elem<DT>::T;
  const int nb = P < kPqsBlocks * 16 ? (P + 15) / 16 : kPqsBlocks;
  const bool vec = (reinterpret_cast<uintptr_t>(q) & 15) == 0 && (a * (int64_t)sizeof(T)) % 16 == 0 &&
                   (b * (int64_t)sizeof(T)) % 16 == 0 && (c * (int64_t)sizeof(T)) % 16 == 0;
  cudaError_t e = vec ? launch_pdl(pqs_part_kernel<DT, D, true>, dim3(nb, L.n_seq), dim3(kPqsThreads), 0, st, L, q, a,
                                   b, c, P, part)
                      : launch_pdl(pqs_part_kernel<DT, D, false>, dim3(nb, L.n_seq), dim3(kPqsThreads), 0, st, L, q,
                                   a, b, c, P, part);
  if (e != cudaSuccess) return e;
  return launch_pdl(pqs_sum_kernel<D>, dim3(L.n_seq), dim3(D), 0, st, (const float*)part, nb, out);
}

cudaError_t launch_prompt_query_sum(const hc_layer& L, const void* q, int64_t a, int64_t b, int64_t c, int P,
                                    float* out, void* scratch, cudaStream_t st) {
  float* part = reinterpret_cast<float*>(scratch);
  HC_DISPATCH_DT_D(L.dtype, L.D, pqs_t, L, q, a, b, c, P, out, part, st);
}

}  // namespace hc
