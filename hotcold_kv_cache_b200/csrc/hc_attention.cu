// Split-K decode attention (flash-decode) for the hot/cold path.
//
// Replaces the reference's Triton kernel evict_fwd_kernel (kernels.py:9-74), which
// runs one program per (batch, query head) over all keys and so reads each KV head
// once per query head of its GQA group. Here one CTA owns (sequence, KV head, chunk
// of CH tokens): its G = Hq/Hk query heads share a single read of the chunk's K and V
// rows, which arrive in shared memory by cp.async.bulk (one 16-byte aligned row copy
// per token, completing on an mbarrier). Scores use 8 lanes per token with 128-bit
// shared loads; each CTA writes a partial (max, sum, output) per query head and the
// last CTA of a (sequence, KV head) to finish merges the partials (counter in global
// memory, reset by that CTA).
//
// Token list of a sequence in slab mode: [held segment (held_len slots) | hot tokens in
// logical order through hot_ord]. Held slot j is attended iff held_valid[j] and
// held_pos[j] <= cur_pos (patch.py:287-289). Dense mode reads (B,Hk,S,D) tensors with a
// (B,S) mask, the drop-in for triton_evict_attention_forward (kernels.py:77-137).
//
// Softmax: the reference exponentiates raw scores (kernels.py:146); it equals the stable
// form computed here except when a logit overflows fp32 exp, where the reference returns
// NaN — reproduced when overflow_nan is set. No unmasked token gives 0/0 = NaN in both.

#include "hc_internal.cuh"

namespace hc {


constexpr int kAttnThreads = 128;
constexpr int kPipeCH = 64;   // rows per chunk of attn_pipe_kernel
constexpr int kPipeSub = 4;   // chunks per CTA of attn_pipe_kernel

template <int DT, int D, int G, int CH>
struct AttnSmem {
  using T = typename Elem<DT>::T;
  static constexpr size_t kOff = 0;
  static constexpr size_t vOff = kOff + sizeof(T) * CH * D;
  static constexpr size_t qOff = vOff + sizeof(T) * CH * D;
  static constexpr size_t sOff = qOff + sizeof(float) * G * D;
  static constexpr size_t mlOff = sOff + sizeof(float) * G * CH;
  static constexpr size_t validOff = mlOff + sizeof(float) * 2 * G;
  static constexpr size_t rowOff = (validOff + sizeof(int) * CH + 15) & ~size_t(15);  // [K|V][CH] row pointers
  static constexpr size_t miscOff = rowOff + 2 * CH * sizeof(void*);
  static constexpr size_t bytes = miscOff + 16;
};

template <int DT, int D, int G, int CH, bool DENSE>
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  using SM = AttnSmem<DT, D, G, CH>;
  constexpr int ROWB = D * sizeof(T);
  constexpr int VEC = 16 / sizeof(T);   // elements per 16-byte load
  constexpr int NJ = D / (8 * VEC);     // 16-byte loads per lane per row (8 lanes per row)
  static_assert(NJ >= 1, "head dim too small");

  extern __shared__ __align__(128) unsigned char smem[];
  T* sK = reinterpret_cast<T*>(smem + SM::kOff);
  T* sV = reinterpret_cast<T*>(smem + SM::vOff);
  float* sQ = reinterpret_cast<float*>(smem + SM::qOff);
  float* sS = reinterpret_cast<float*>(smem + SM::sOff);
  float* sML = reinterpret_cast<float*>(smem + SM::mlOff);
  int* sValid = reinterpret_cast<int*>(smem + SM::validOff);
  const T** sRow = reinterpret_cast<const T**>(smem + SM::rowOff);
  int* sMisc = reinterpret_cast<int*>(smem + SM::miscOff);
  constexpr int CPR = D / VEC;  // 16-byte chunks per row

  const int c = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  pdl_wait();

  // ---- token range of this chunk -------------------------------------------------------
  int n_held = 0, n_tok;
  hc_seq_desc d;
  hc_seq_state* st = nullptr;
  if constexpr (DENSE) {
    n_tok = a.S;
  } else {
    d = a.desc[s];
    st = d.st;
    n_held = a.use_held ? max(0, min(st->held_len, d.r_max)) : 0;
    n_tok = n_held + max(0, min(st->n_hot, d.cap));
  }
  const int n_chunks = (n_tok + CH - 1) / CH;
  if (c >= n_chunks) return;
  const int t0 = c * CH;
  const int nt = min(CH, n_tok - t0);

  // ---- resolve rows, then gather them with 16-byte cp.async (K and V in two groups) --------
  const T* krow = nullptr;
  const T* vrow = nullptr;
  bool copy = false;
  if (tid < nt) {
    const int t = t0 + tid;
    int valid = 1;
    if constexpr (DENSE) {
      const size_t off = (((size_t)s * a.Hk + h) * a.S + t) * D;
      krow = reinterpret_cast<const T*>(a.k) + off;
      vrow = reinterpret_cast<const T*>(a.v) + off;
      valid = a.mask[(size_t)s * a.S + t] != 0;
      copy = true;
    } else if (t < n_held) {
      const size_t off = ((size_t)h * d.r_max + t) * D;
      krow = reinterpret_cast<const T*>(d.held_k) + off;
      vrow = reinterpret_cast<const T*>(d.held_v) + off;
      valid = d.held_valid[t] != 0 && d.held_pos[t] <= a.cur_pos[s];
      copy = true;
    } else {
      const int slot = d.hot_ord[t - n_held];
      if (slot >= 0 && slot < d.cap) {
        const size_t off = ((size_t)h * d.cap + slot) * D;
        krow = reinterpret_cast<const T*>(d.hot_k) + off;
        vrow = reinterpret_cast<const T*>(d.hot_v) + off;
        copy = true;
      } else {
        valid = 0;
        set_status(st, HC_DEV_INDEX);
      }
    }
    sValid[tid] = valid;
  }
  if (tid < CH) {
    sRow[tid] = copy ? krow : nullptr;
    sRow[CH + tid] = copy ? vrow : nullptr;
  }
  __syncthreads();
  // rows without a source (and rows past the chunk) read as zeros
  for (int k = tid; k < nt * CPR; k += kAttnThreads) {
    const int r = k / CPR, q = k % CPR;
    const T* kr = sRow[r];
    cp_async16(sK + (size_t)r * D + q * VEC, kr ? kr + q * VEC : reinterpret_cast<const T*>(a.q), kr ? 16 : 0);
  }
  cp_async_commit();
  for (int k = tid; k < nt * CPR; k += kAttnThreads) {
    const int r = k / CPR, q = k % CPR;
    const T* vr = sRow[CH + r];
    cp_async16(sV + (size_t)r * D + q * VEC, vr ? vr + q * VEC : reinterpret_cast<const T*>(a.q), vr ? 16 : 0);
  }
  cp_async_commit();
  // query heads of this KV head -> shared (float), while the rows are in flight
  const T* qg = reinterpret_cast<const T*>(a.q) + ((size_t)s * a.Hq + (size_t)h * G) * D;
  for (int i = tid; i < G * D; i += kAttnThreads) sQ[i] = E::to_f(qg[i]);
  __syncthreads();
  // q fragments in registers: lane `sub` owns d = j*8*VEC + sub*VEC + e
  const int sub = lane & 7, tk = lane >> 3;
  float qr[G][NJ * VEC];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < VEC; ++e) qr[g][j * VEC + e] = sQ[g * D + j * 8 * VEC + sub * VEC + e];

  cp_async_wait<1>();  // K rows landed (V may still be in flight)
  __syncthreads();

  // ---- scores: 4 tokens per warp per pass, 8 lanes per token ----------------------------
  for (int base = warp * 4; base < nt; base += 16) {
    const int t = base + tk;
    float acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = 0.f;
    if (t < nt) {
      const T* row = sK + (size_t)t * D;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        uint4 u = *reinterpret_cast<const uint4*>(row + j * 8 * VEC + sub * VEC);
        float kf[VEC];
        unpack16<DT>(u, kf);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[g] = fmaf(qr[g][j * VEC + e], kf[e], acc[g]);
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 4);
      acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
      acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
    }
    if (sub == 0 && t < nt) {
#pragma unroll
      for (int g = 0; g < G; ++g) sS[g * CH + t] = sValid[t] ? acc[g] * a.scale : kNegInf;
    }
  }
  __syncthreads();

  // ---- chunk softmax statistics, probabilities in place ---------------------------------
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float m = kNegInf;
    for (int t = lane; t < nt; t += 32) m = fmaxf(m, sS[g * CH + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float x = sS[g * CH + t];
      const float p = (x == kNegInf) ? 0.f : __expf(x - m);
      sS[g * CH + t] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sML[g] = m;
      sML[G + g] = l;
    }
  }
  cp_async_wait<0>();  // V rows landed
  __syncthreads();

  // ---- P.V: thread d owns output column d for every query head ----------------------------
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) o[g] = 0.f;
  if (tid < D) {
    for (int t = 0; t < nt; ++t) {
      const float vv = E::to_f(sV[(size_t)t * D + tid]);
#pragma unroll
      for (int g = 0; g < G; ++g) o[g] = fmaf(sS[g * CH + t], vv, o[g]);
    }
  }

  const size_t head0 = (size_t)s * a.Hq + (size_t)h * G;
  T* outp = reinterpret_cast<T*>(a.out);
  if (n_chunks == 1) {
    if (tid < D) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float r = o[g] / sML[G + g];
        if (a.overflow_nan && sML[g] >= kExpOverflow) r = __int_as_float(0x7fc00000);
        outp[(head0 + g) * D + tid] = E::from_f(r);
      }
    }
    if (a.ml && tid < G) {
      a.ml[(head0 + tid) * 2] = sML[tid];
      a.ml[(head0 + tid) * 2 + 1] = sML[G + tid];
    }
    pdl_launch_dependents();
    return;
  }

  // ---- partials, then the last CTA of this (sequence, KV head) merges them ---------------
  constexpr int PSTRIDE = G * D + 2 * G;
  float* pbase = a.part + ((size_t)s * a.Hk + h) * (size_t)a.max_chunks * PSTRIDE;
  float* mine = pbase + (size_t)c * PSTRIDE;
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < G; ++g) mine[g * D + tid] = o[g];
  }
  if (tid < 2 * G) mine[G * D + tid] = sML[tid];
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&a.counters[(size_t)s * a.Hk + h], 1);
    sMisc[0] = (prev == n_chunks - 1);
  }
  __syncthreads();
  if (!sMisc[0]) return;
  __threadfence();
  if (tid == 0) a.counters[(size_t)s * a.Hk + h] = 0;

  // per query head: the overall max and sum from the chunks' (max, sum), a warp per head with
  // its lanes over the chunks; then every output column as a weighted sum of the partials,
  // eight chunks' loads in flight per thread
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float M = kNegInf;
    for (int cc = lane; cc < n_chunks; cc += 32) M = fmaxf(M, __ldcg(pbase + (size_t)cc * PSTRIDE + G * D + g));
    M = warp_max(M);
    float L = 0.f;
    for (int cc = lane; cc < n_chunks; cc += 32) {
      const float* pc = pbase + (size_t)cc * PSTRIDE;
      L = fmaf(__ldcg(pc + G * D + G + g), __expf(__ldcg(pc + G * D + g) - M), L);
    }
    L = warp_sum(L);
    if (lane == 0) {
      sML[g] = M;
      sML[G + g] = L;
    }
  }
  __syncthreads();
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float M = sML[g], L = sML[G + g];
      float O = 0.f;
      int cc = 0;
      for (; cc + 8 <= n_chunks; cc += 8) {
        float x[8], m[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float* pc = pbase + (size_t)(cc + u) * PSTRIDE;
          x[u] = __ldcg(pc + g * D + tid);
          m[u] = __ldcg(pc + G * D + g);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) O = fmaf(x[u], __expf(m[u] - M), O);
      }
      for (; cc < n_chunks; ++cc) {
        const float* pc = pbase + (size_t)cc * PSTRIDE;
        O = fmaf(__ldcg(pc + g * D + tid), __expf(__ldcg(pc + G * D + g) - M), O);
      }
      float r = O / L;
      if (a.overflow_nan && M >= kExpOverflow) r = __int_as_float(0x7fc00000);
      outp[(head0 + g) * D + tid] = E::from_f(r);
      if (a.ml && tid == 0) {
        a.ml[(head0 + g) * 2] = M;
        a.ml[(head0 + g) * 2 + 1] = L;
      }
    }
  }
  pdl_launch_dependents();
}

// Slab attention for large batches: CTA (c, h, s) covers NSUB consecutive chunks of CH rows
// ([held | hot] order) with two buffers, so the bulk copies of chunk j + 1 land while chunk j is
// scored; the softmax is carried across the chunks online (running max, sum and a rescale of
// the partial output), then the CTA's partial is merged as in attn_kernel.
template <int DT, int D, int G, int CH>
struct PipeSmem {
  using T = typename Elem<DT>::T;
  static constexpr size_t kOff = 0;                                    // [2][CH][D]
  static constexpr size_t vOff = kOff + 2 * sizeof(T) * CH * D;        // [2][CH][D]
  static constexpr size_t qOff = vOff + 2 * sizeof(T) * CH * D;        // [G][D] fp32
  static constexpr size_t sOff = qOff + sizeof(float) * G * D;         // [G][CH] scores, then p
  static constexpr size_t mlOff = sOff + sizeof(float) * G * CH;       // running max [G], sum [G], rescale [G]
  static constexpr size_t validOff = mlOff + sizeof(float) * 3 * G;    // [2][CH]
  static constexpr size_t rowOff = (validOff + sizeof(int) * 2 * CH + 15) & ~size_t(15);  // [2][2][CH] row pointers
  static constexpr size_t miscOff = rowOff + 2 * 2 * CH * sizeof(void*);
  static constexpr size_t bytes = miscOff + 16;
};

template <int DT, int D, int G, int CH, int NSUB>
__global__ void __launch_bounds__(kAttnThreads) attn_pipe_kernel(AttnArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  using SM = PipeSmem<DT, D, G, CH>;
  constexpr int VEC = 16 / sizeof(T);
  constexpr int NJ = D / (8 * VEC);
  constexpr int CPR = D / VEC;  // 16-byte chunks per row
  constexpr int SPAN = CH * NSUB;
  extern __shared__ __align__(128) unsigned char smem[];
  T* sK = reinterpret_cast<T*>(smem + SM::kOff);
  T* sV = reinterpret_cast<T*>(smem + SM::vOff);
  float* sQ = reinterpret_cast<float*>(smem + SM::qOff);
  float* sS = reinterpret_cast<float*>(smem + SM::sOff);
  float* sML = reinterpret_cast<float*>(smem + SM::mlOff);
  int* sValid = reinterpret_cast<int*>(smem + SM::validOff);
  const T** sRow = reinterpret_cast<const T**>(smem + SM::rowOff);  // [buf][K|V][CH]
  int* sMisc = reinterpret_cast<int*>(smem + SM::miscOff);

  const int c = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  const hc_seq_desc d = a.desc[s];
  hc_seq_state* st = d.st;
  const int n_held = a.use_held ? max(0, min(st->held_len, d.r_max)) : 0;
  const int n_tok = n_held + max(0, min(st->n_hot, d.cap));
  const int n_chunks = (n_tok + SPAN - 1) / SPAN;
  if (c >= n_chunks) return;
  const int base0 = c * SPAN;
  const int nsub = min(NSUB, (n_tok - base0 + CH - 1) / CH);
  if (tid < G) {
    sML[tid] = kNegInf;
    sML[G + tid] = 0.f;
  }

  // rows of chunk j into buffer j & 1 with 16-byte cp.async gathers (one commit group per chunk);
  // an out-of-range slot is reported and its row reads as zeros
  auto stage = [&](int j) {
    const int buf = j & 1;
    const int t0 = base0 + j * CH, nt = min(CH, n_tok - t0);
    T* bk = sK + (size_t)buf * CH * D;
    T* bv = sV + (size_t)buf * CH * D;
    const T** rk = sRow + (size_t)buf * 2 * CH;
    const T** rv = rk + CH;
    if (tid < CH) {
      const T* krow = nullptr;
      const T* vrow = nullptr;
      int valid = 0;
      if (tid < nt) {
        const int t = t0 + tid;
        valid = 1;
        if (t < n_held) {
          const size_t off = ((size_t)h * d.r_max + t) * D;
          krow = reinterpret_cast<const T*>(d.held_k) + off;
          vrow = reinterpret_cast<const T*>(d.held_v) + off;
          valid = d.held_valid[t] != 0 && d.held_pos[t] <= a.cur_pos[s];
        } else {
          const int slot = d.hot_ord[t - n_held];
          if (slot >= 0 && slot < d.cap) {
            const size_t off = ((size_t)h * d.cap + slot) * D;
            krow = reinterpret_cast<const T*>(d.hot_k) + off;
            vrow = reinterpret_cast<const T*>(d.hot_v) + off;
          } else {
            valid = 0;
            set_status(st, HC_DEV_INDEX);
          }
        }
      }
      rk[tid] = krow;
      rv[tid] = vrow;
      sValid[buf * CH + tid] = valid;
    }
    __syncthreads();
    for (int k = tid; k < CH * CPR; k += kAttnThreads) {
      const int r = k / CPR, q = k % CPR;
      const T* kr = rk[r];
      const T* vr = rv[r];
      cp_async16(bk + (size_t)r * D + q * VEC, kr ? kr + q * VEC : reinterpret_cast<const T*>(a.q), kr ? 16 : 0);
      cp_async16(bv + (size_t)r * D + q * VEC, vr ? vr + q * VEC : reinterpret_cast<const T*>(a.q), vr ? 16 : 0);
    }
    cp_async_commit();
  };

  stage(0);
  if (nsub > 1) stage(1);
  const T* qg = reinterpret_cast<const T*>(a.q) + ((size_t)s * a.Hq + (size_t)h * G) * D;
  for (int i = tid; i < G * D; i += kAttnThreads) sQ[i] = E::to_f(qg[i]);
  __syncthreads();
  const int sub = lane & 7, tk = lane >> 3;
  float qr[G][NJ * VEC];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < VEC; ++e) qr[g][j * VEC + e] = sQ[g * D + j * 8 * VEC + sub * VEC + e];
  // P.V: thread (row group grp, column chunk cc) accumulates 16-byte column chunk cc of every
  // query head over rows grp, grp + NGRP, ... (packed fp32 FMAs); the groups are added at the end
  constexpr int KCH = D / VEC;               // 16-byte column chunks per row
  constexpr int NGRP = kAttnThreads / KCH;   // row groups
  const int cch = tid % KCH, grp = tid / KCH;
  float2 o2[G][VEC / 2];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < VEC / 2; ++e) o2[g][e] = make_float2(0.f, 0.f);

  for (int j = 0; j < nsub; ++j) {
    const int buf = j & 1;
    const int nt = min(CH, n_tok - (base0 + j * CH));
    const T* bk = sK + (size_t)buf * CH * D;
    const T* bv = sV + (size_t)buf * CH * D;
    const int* bval = sValid + buf * CH;
    if (j + 1 < nsub) cp_async_wait<1>();  // chunk j landed, chunk j + 1 may still be in flight
    else cp_async_wait<0>();
    __syncthreads();
    for (int b4 = warp * 4; b4 < nt; b4 += 16) {
      const int t = b4 + tk;
      float acc[G];
      float2 acc2[G];  // packed fp32 FMAs over element pairs, the pair added at the end
#pragma unroll
      for (int g = 0; g < G; ++g) acc2[g] = make_float2(0.f, 0.f);
      if (t < nt) {
        const T* row = bk + (size_t)t * D;
#pragma unroll
        for (int jj = 0; jj < NJ; ++jj) {
          uint4 u = *reinterpret_cast<const uint4*>(row + jj * 8 * VEC + sub * VEC);
          float kf[VEC];
          unpack16<DT>(u, kf);
#pragma unroll
          for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < VEC; e += 2)
              acc2[g] = __ffma2_rn(make_float2(qr[g][jj * VEC + e], qr[g][jj * VEC + e + 1]),
                                   make_float2(kf[e], kf[e + 1]), acc2[g]);
        }
      }
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = acc2[g].x + acc2[g].y;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 4);
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
      }
      if (sub == 0 && t < nt) {
#pragma unroll
        for (int g = 0; g < G; ++g) sS[g * CH + t] = bval[t] ? acc[g] * a.scale : kNegInf;
      }
    }
    __syncthreads();
    // online softmax: the chunk's probabilities against the running max, and the factor that
    // rescales what was accumulated before
    for (int g = warp; g < G; g += kAttnThreads / 32) {
      float mc = kNegInf;
      for (int t = lane; t < nt; t += 32) mc = fmaxf(mc, sS[g * CH + t]);
      mc = warp_max(mc);
      const float m_old = sML[g];
      const float m_new = fmaxf(m_old, mc);
      float l = 0.f;
      for (int t = lane; t < nt; t += 32) {
        const float x = sS[g * CH + t];
        const float pr = (x == kNegInf) ? 0.f : __expf(x - m_new);
        sS[g * CH + t] = pr;
        l += pr;
      }
      l = warp_sum(l);
      __syncwarp();
      if (lane == 0) {
        const float alpha = (m_old == kNegInf) ? 0.f : __expf(m_old - m_new);
        sML[g] = m_new;
        sML[G + g] = sML[G + g] * alpha + l;
        sML[2 * G + g] = alpha;
      }
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float al = sML[2 * G + g];
      const float2 a2 = make_float2(al, al);
#pragma unroll
      for (int e = 0; e < VEC / 2; ++e) o2[g][e] = __fmul2_rn(o2[g][e], a2);
    }
    for (int t = grp; t < nt; t += NGRP) {
      float vf[VEC];
      unpack16<DT>(*reinterpret_cast<const uint4*>(bv + (size_t)t * D + cch * VEC), vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = sS[g * CH + t];
        const float2 p2 = make_float2(pr, pr);
#pragma unroll
        for (int e = 0; e < VEC / 2; ++e) o2[g][e] = __ffma2_rn(p2, make_float2(vf[2 * e], vf[2 * e + 1]), o2[g][e]);
      }
    }
    __syncthreads();  // buffer `buf` and the scores are free
    if (j + 2 < nsub) stage(j + 2);
  }

  // the row groups' column chunks, added per column (the key and value buffers, contiguous, are
  // free: no copy is in flight after the last chunk)
  float* red = reinterpret_cast<float*>(sK);  // [NGRP][G][D] fp32 over the key and value buffers
  static_assert((size_t)NGRP * G * D * 4 <= 4 * sizeof(T) * CH * D, "reduction buffer");
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int e = 0; e < VEC / 2; ++e)
      *reinterpret_cast<float2*>(red + ((size_t)grp * G + g) * D + cch * VEC + 2 * e) = o2[g][e];
  __syncthreads();
  float o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    o[g] = 0.f;
    if (tid < D)
#pragma unroll
      for (int q = 0; q < NGRP; ++q) o[g] += red[((size_t)q * G + g) * D + tid];
  }
  const size_t head0 = (size_t)s * a.Hq + (size_t)h * G;
  T* outp = reinterpret_cast<T*>(a.out);
  if (n_chunks == 1) {
    if (tid < D) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float r = o[g] / sML[G + g];
        if (a.overflow_nan && sML[g] >= kExpOverflow) r = __int_as_float(0x7fc00000);
        outp[(head0 + g) * D + tid] = E::from_f(r);
      }
    }
    pdl_launch_dependents();
    return;
  }
  constexpr int PSTRIDE = G * D + 2 * G;
  float* pbase = a.part + ((size_t)s * a.Hk + h) * (size_t)a.max_chunks * PSTRIDE;
  float* mine = pbase + (size_t)c * PSTRIDE;
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < G; ++g) mine[g * D + tid] = o[g];
  }
  if (tid < 2 * G) mine[G * D + tid] = sML[tid];
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(&a.counters[(size_t)s * a.Hk + h], 1);
    sMisc[0] = (prev == n_chunks - 1);
  }
  __syncthreads();
  if (!sMisc[0]) return;
  __threadfence();
  if (tid == 0) a.counters[(size_t)s * a.Hk + h] = 0;
  for (int g = warp; g < G; g += kAttnThreads / 32) {
    float M = kNegInf;
    for (int cc = lane; cc < n_chunks; cc += 32) M = fmaxf(M, __ldcg(pbase + (size_t)cc * PSTRIDE + G * D + g));
    M = warp_max(M);
    float L = 0.f;
    for (int cc = lane; cc < n_chunks; cc += 32) {
      const float* pc = pbase + (size_t)cc * PSTRIDE;
      L = fmaf(__ldcg(pc + G * D + G + g), __expf(__ldcg(pc + G * D + g) - M), L);
    }
    L = warp_sum(L);
    __syncwarp();
    if (lane == 0) {
      sML[g] = M;
      sML[G + g] = L;
    }
  }
  __syncthreads();
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float M = sML[g], L = sML[G + g];
      float O = 0.f;
      for (int cc = 0; cc < n_chunks; ++cc) {
        const float* pc = pbase + (size_t)cc * PSTRIDE;
        O = fmaf(__ldcg(pc + g * D + tid), __expf(__ldcg(pc + G * D + g) - M), O);
      }
      float r = O / L;
      if (a.overflow_nan && M >= kExpOverflow) r = __int_as_float(0x7fc00000);
      outp[(head0 + g) * D + tid] = E::from_f(r);
    }
  }
  pdl_launch_dependents();
}

// Second output of the dense drop-in (kernels.py:103,134-137): per token the mean over query
// heads of softmax probability times sum_d |v_d| / D, rounded to the input dtype; masked
// tokens contribute exactly 0 (the reference's exp(-1e35)).
// The wrapper's second result (kernels.py:134-137): loss[t] = mean over query heads of
// softmax(q.k)[t] * sum_d |v[t]| / D, cast to the input dtype, then its argmin (first index on
// ties, argmin_kernel). A CTA takes 32 tokens of one sequence with a warp per KV head and a lane
// per token: the head group's query rows and final softmax statistics (written by the attention
// kernel) sit in shared memory, so a lane reads its token's K and V rows once and needs no
// cross-lane reductions; the per-head terms are summed in head order through shared memory.
constexpr int kLossTok = 32;

template <int DT, int D, int G>
__global__ void __launch_bounds__(256) evict_loss_kernel(const void* q_, const void* k_, const void* v_,
                                                         const uint8_t* mask, const float* ml, float* loss, int Hq,
                                                         int Hk, int S, float scale) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VE = 16 / sizeof(T);  // elements per 16-byte chunk
  constexpr int NC = D / VE;          // chunks per row
  extern __shared__ float sq[];       // [Hq][D] query rows, [Hq][2] (max, sum), [Hk][kLossTok] terms
  float* sml = sq + (size_t)Hq * D;
  float* sterm = sml + 2 * (size_t)Hq;
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  pdl_wait();
  const T* q = reinterpret_cast<const T*>(q_) + (size_t)b * Hq * D;
  for (int i = threadIdx.x; i < Hq * D; i += blockDim.x) sq[i] = E::to_f(q[i]);
  for (int i = threadIdx.x; i < Hq; i += blockDim.x) {
    sml[2 * i] = ml[((size_t)b * Hq + i) * 2];
    sml[2 * i + 1] = ml[((size_t)b * Hq + i) * 2 + 1];
  }
  __syncthreads();
  const int t = blockIdx.x * kLossTok + lane;
  const bool live = t < S;
  const bool m = live && mask[(size_t)b * S + t] != 0;
  for (int h = warp; h < Hk; h += nw) {
    float term = 0.f;
    if (live) {
      const uint4* kr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(k_) + (((size_t)b * Hk + h) * S + t) * D);
      const uint4* vr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(v_) + (((size_t)b * Hk + h) * S + t) * D);
      float dot[G];
#pragma unroll
      for (int g = 0; g < G; ++g) dot[g] = 0.f;
      float av = 0.f;
#pragma unroll 4
      for (int c = 0; c < NC; ++c) {
        float kf[VE], vf[VE];
        unpack16<DT>(kr[c], kf);
        unpack16<DT>(vr[c], vf);
#pragma unroll
        for (int e = 0; e < VE; ++e) av += fabsf(vf[e]);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float* qg = sq + (size_t)(h * G + g) * D + c * VE;
#pragma unroll
          for (int e = 0; e < VE; ++e) dot[g] = fmaf(qg[e], kf[e], dot[g]);
        }
      }
      av /= (float)D;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const int hq = h * G + g;
        const float p = m ? __expf(dot[g] * scale - sml[2 * hq]) / sml[2 * hq + 1] : 0.f;
        term += p * av;
      }
    }
    sterm[h * kLossTok + lane] = term;
  }
  __syncthreads();
  if (threadIdx.x < kLossTok && t < S) {
    float acc = 0.f;
    for (int h = 0; h < Hk; ++h) acc += sterm[h * kLossTok + threadIdx.x];
    loss[(size_t)b * S + t] = E::round(acc / (float)Hq);
  }
}

__global__ void __launch_bounds__(1024) argmin_kernel(const float* loss, int S, int64_t* out) {
  const int b = blockIdx.x;
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_wait();
  float best = __int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  for (int t = threadIdx.x; t < S; t += blockDim.x) {
    const float x = loss[(size_t)b * S + t];
    if (x < best || (x == best && t < bi)) {
      best = x;
      bi = t;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob < best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] < best || (sv[w] == best && si[w] < bi)) {
        best = sv[w];
        bi = si[w];
      }
    out[b] = bi == 0x7fffffff ? 0 : bi;
  }
}

// ------------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------------
template <int DT, int D, int G, int CH, bool DENSE>
cudaError_t launch_attn_t(const AttnArgs& a, int n_seq, cudaStream_t stream) {
  using SM = AttnSmem<DT, D, G, CH>;
  auto kern = attn_kernel<DT, D, G, CH, DENSE>;
  cudaError_t e = ensure_smem(kern, SM::bytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.max_chunks, a.Hk, n_seq);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = SM::bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int DT, int D, int CH, bool DENSE>
cudaError_t launch_attn_g(const AttnArgs& a, int G, int n_seq, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_attn_t<DT, D, 1, CH, DENSE>(a, n_seq, stream);
    case 2: return launch_attn_t<DT, D, 2, CH, DENSE>(a, n_seq, stream);
    case 4: return launch_attn_t<DT, D, 4, CH, DENSE>(a, n_seq, stream);
    case 8: return launch_attn_t<DT, D, 8, CH, DENSE>(a, n_seq, stream);
  }
  return cudaErrorInvalidValue;
}

template <int DT, bool DENSE>
cudaError_t launch_attn_d(const AttnArgs& a, int D, int G, int CH, int n_seq, cudaStream_t stream) {
  if (D == 128) {
    if (CH == 32) return launch_attn_g<DT, 128, 32, DENSE>(a, G, n_seq, stream);
    return launch_attn_g<DT, 128, 64, DENSE>(a, G, n_seq, stream);
  }
  if (D == 64) {
    if (CH == 32) return launch_attn_g<DT, 64, 32, DENSE>(a, G, n_seq, stream);
    return launch_attn_g<DT, 64, 64, DENSE>(a, G, n_seq, stream);
  }
  return cudaErrorInvalidValue;
}

// Chunk length: 32 tokens when the whole batch would otherwise fill fewer than ~2 waves
// of 148 SMs, else 64.
int attn_chunk(int n_seq, int Hk, int max_tokens) {
  const long ctas64 = (long)n_seq * Hk * ((max_tokens + 63) / 64);
  return ctas64 < 296 ? 32 : 64;
}

template <int DT, int D, int G>
cudaError_t launch_pipe_t(const AttnArgs& a, int n_seq, cudaStream_t stream) {
  using SM = PipeSmem<DT, D, G, kPipeCH>;
  auto kern = attn_pipe_kernel<DT, D, G, kPipeCH, kPipeSub>;
  cudaError_t e = ensure_smem(kern, SM::bytes);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.max_chunks, a.Hk, n_seq);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = SM::bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int DT, int D>
cudaError_t launch_pipe_g(const AttnArgs& a, int G, int n_seq, cudaStream_t stream) {
  switch (G) {
    case 1: return launch_pipe_t<DT, D, 1>(a, n_seq, stream);
    case 2: return launch_pipe_t<DT, D, 2>(a, n_seq, stream);
    case 4: return launch_pipe_t<DT, D, 4>(a, n_seq, stream);
    case 8: return launch_pipe_t<DT, D, 8>(a, n_seq, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_attention(const AttnArgs& a0, int dtype, int D, int G, int n_seq, int max_tokens, bool dense,
                             cudaStream_t stream) {
  AttnArgs a = a0;
  const long pipe_ctas = (long)n_seq * a.Hk * ((max_tokens + kPipeCH * kPipeSub - 1) / (kPipeCH * kPipeSub));
  if (!dense && pipe_ctas >= 2 * 148 && max_tokens > kPipeCH * kPipeSub) {
    // large slab batches: four chunks per CTA, copies of the next chunk overlapping the math
    a.max_chunks = (max_tokens + kPipeCH * kPipeSub - 1) / (kPipeCH * kPipeSub);
#define HC_PIPE(DTV, DV) \
    if (dtype == DTV && D == DV) return launch_pipe_g<DTV, DV>(a, G, n_seq, stream);
    HC_PIPE(HC_F32, 128) HC_PIPE(HC_F16, 128) HC_PIPE(HC_BF16, 128)
    HC_PIPE(HC_F32, 64) HC_PIPE(HC_F16, 64) HC_PIPE(HC_BF16, 64)
#undef HC_PIPE
    return cudaErrorInvalidValue;
  }
  const int CH = attn_chunk(n_seq, a.Hk, max_tokens);
  a.max_chunks = (max_tokens + CH - 1) / CH;
  if (a.max_chunks < 1) a.max_chunks = 1;
  if (dense) {
    switch (dtype) {
      case HC_F32: return launch_attn_d<HC_F32, true>(a, D, G, CH, n_seq, stream);
      case HC_F16: return launch_attn_d<HC_F16, true>(a, D, G, CH, n_seq, stream);
      case HC_BF16: return launch_attn_d<HC_BF16, true>(a, D, G, CH, n_seq, stream);
    }
  } else {
    switch (dtype) {
      case HC_F32: return launch_attn_d<HC_F32, false>(a, D, G, CH, n_seq, stream);
      case HC_F16: return launch_attn_d<HC_F16, false>(a, D, G, CH, n_seq, stream);
      case HC_BF16: return launch_attn_d<HC_BF16, false>(a, D, G, CH, n_seq, stream);
    }
  }
  return cudaErrorInvalidValue;
}

size_t attention_part_bytes(int n_seq, int Hq, int Hk, int D, int max_tokens) {
  const int G = Hq / Hk;
  const size_t chunks = (size_t)(max_tokens + 31) / 32 + 1;
  return (size_t)n_seq * Hk * chunks * (size_t)(G * D + 2 * G) * sizeof(float);
}

template <int DT, int D, int G>
cudaError_t launch_loss_t(const void* q, const void* k, const void* v, const uint8_t* mask, const float* ml,
                          float* loss, int64_t* out, int B, int Hq, int Hk, int S, float scale, cudaStream_t stream) {
  auto kern = evict_loss_kernel<DT, D, G>;
  const size_t smem = ((size_t)Hq * D + 2 * (size_t)Hq + (size_t)Hk * kLossTok) * sizeof(float);
  cudaError_t e = ensure_smem(kern, smem);
  if (e != cudaSuccess) return e;
  const int warps = Hk < 8 ? Hk : 8;
  e = launch_pdl(kern, dim3((S + kLossTok - 1) / kLossTok, B), dim3(32 * warps), smem, stream, q, k, v, mask, ml, loss,
                 Hq, Hk, S, scale);
  if (e != cudaSuccess) return e;
  return launch_pdl(argmin_kernel, dim3(B), dim3(1024), 0, stream, (const float*)loss, S, out);
}

cudaError_t launch_evict_idx(int dtype, const void* q, const void* k, const void* v, const uint8_t* mask,
                             const float* ml, float* loss, int64_t* out, int B, int Hq, int Hk, int S, int D,
                             float scale, cudaStream_t stream) {
  const int G = Hq / Hk;
#define HC_LOSS_CASE(DTV, DV, GV) \
  if (dtype == DTV && D == DV && G == GV) return launch_loss_t<DTV, DV, GV>(q, k, v, mask, ml, loss, out, B, Hq, Hk, S, scale, stream);
#define HC_LOSS_G(DTV, DV) HC_LOSS_CASE(DTV, DV, 1) HC_LOSS_CASE(DTV, DV, 2) HC_LOSS_CASE(DTV, DV, 4) HC_LOSS_CASE(DTV, DV, 8)
  HC_LOSS_G(HC_F32, 128) HC_LOSS_G(HC_F16, 128) HC_LOSS_G(HC_BF16, 128)
  HC_LOSS_G(HC_F32, 64) HC_LOSS_G(HC_F16, 64) HC_LOSS_G(HC_BF16, 64)
#undef HC_LOSS_G
#undef HC_LOSS_CASE
  return cudaErrorInvalidValue;
}

}  // namespace hc
