// Fused decode step of one layer: append, compression with eviction into the cold ring, and
// attention over [held | hot] in one launch — one thread-block cluster of 16 CTAs per sequence.
//
// The reference runs this as a chain of torch ops and a Triton kernel per layer
// (patch.py:161-305 with cache.py:130-151 and cache.py:37-128). Split into separate kernels
// (hc_append, hc_compress, hc_attend) the step pays a launch and a global round trip per
// stage; at batch 1 that latency, not HBM bandwidth, sets the time. Here CTA (h, p) of the
// cluster owns KV head h and part p of P = 16/Hk parts:
//   1. it gathers (cp.async, 16-byte chunks) the K rows of its 1/P of the token list
//      [held | hot | new] and the V columns p*D/P .. (p+1)*D/P of every token, RoPEs the new
//      token's query heads of its group (and, if the new token is its own, the key), and scores
//      its tokens on the tensor cores: one m16n8k16 MMA tile row per query head plus a row
//      for the GQA-mean query, whose product is the eviction logit;
//   2. attention logits go to the other CTAs of head h and eviction logits to every CTA
//      through distributed shared memory (cluster barrier 1);
//   3. every CTA applies the policy to all hot tokens (hot/cold sum, or SnapKV softmax +
//      pooling + head mean), ranks the tokens of its own 32-token words against the whole
//      prefix (exact top-k, ties to the lower index) and publishes their eviction bits and
//      counts (cluster barrier 2); there is no leader CTA on the critical path;
//   4. every CTA masks the evicted tokens, takes the softmax over all tokens of head h and
//      writes its D/P output columns; the owners of each word compact the logical order,
//      push freed slots and copy evicted payloads into the cold ring with their index vectors.
// The result equals hc_append + hc_compress + hc_attend on the same state.

#include <cooperative_groups.h>

#include "hc_internal.cuh"

namespace cg = cooperative_groups;

namespace hc {

constexpr int kStepThreads = 512;
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepMaxCluster = 16;

// Sizes shared by the host and the kernel.
struct StepGeom {
  int P;     // parts per KV head; cluster = Hk * P = 16
  int tpc;   // scored rows per CTA (multiple of 8)
  int tmax;  // tokens of [held | hot] at most (multiple of 8)
  int s_cap; // hot tokens at most
  int wpc;   // 32-token words a CTA owns at most
  int dpc;   // V columns per CTA
};

__host__ __device__ inline StepGeom step_geom(int Hk, int D, int max_cap, int max_r, int use_held) {
  StepGeom g{};
  g.P = (Hk >= 1 && Hk <= kStepMaxCluster && kStepMaxCluster % Hk == 0) ? kStepMaxCluster / Hk : 0;
  if (!g.P) return g;
  g.s_cap = max_cap;
  g.tmax = ((use_held ? max_r : 0) + max_cap + 7) & ~7;
  g.tpc = (((g.tmax + g.P - 1) / g.P) + 7) & ~7;
  g.wpc = ((max_cap + 31) / 32 + kStepMaxCluster - 1) / kStepMaxCluster;
  g.dpc = D / g.P;
  return g;
}

struct StepArgs {
  hc_layer L;
  const void* q_pre;
  int64_t qss;
  const void* k_pre;
  const void* v;
  int64_t kvss;
  const void* cos;
  const void* sin;
  const int64_t* pos;
  void* out;
  int use_held, overflow_nan;
  StepGeom g;
};

struct StepSmem {
  size_t k, v, qh, q, a, ord, fre, held, e, pool, key, red, best, mask, cnt, word, flag, evl, misc, total;
};

__host__ __device__ inline size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline StepSmem step_smem(int D, int esz, int G, int Hk, const StepGeom& g) {
  StepSmem m{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t r = o; o += al16(b); return r; };
  // K rows of this CTA's tokens; after scoring the same area holds the P.V partial sums
  const size_t kb = (size_t)g.tpc * D * esz;
  const size_t rb = (size_t)kStepWarps * G * (g.dpc + 1) * 4;
  m.k = take(kb > rb ? kb : rb);
  m.v = take((size_t)g.tmax * g.dpc * esz);
  m.qh = take((size_t)16 * (D + 8) * esz);   // MMA query operand: G heads, the mean, zero rows
  m.q = take((size_t)(G + 1) * D * 4);
  m.a = take((size_t)G * g.tmax * 4);        // attention logits, then probabilities
  m.ord = take((size_t)g.s_cap * 4);         // logical order (physical slot per logical index)
  m.fre = take((size_t)g.s_cap * 4);         // free-slot stack
  m.held = take((size_t)g.tmax * 4);         // held rows attended this step
  m.e = take((size_t)g.tmax * 4);            // eviction logits of head h, by token index
  m.pool = take((size_t)Hk * g.wpc * 32 * 4);  // per-head policy values of the tokens this CTA owns
  m.key = take((size_t)g.s_cap * 4);         // policy score keys, by logical index
  m.red = take((size_t)(4 * kStepMaxCluster + 4 * kStepWarps) * 8);
  m.best = take((size_t)kStepMaxCluster * 8);
  m.mask = take((size_t)((g.s_cap + 31) / 32) * 4);
  m.cnt = take((size_t)2 * kStepMaxCluster * 4);
  m.word = take((size_t)g.wpc * 4);
  m.flag = take((size_t)g.wpc * 32 * 4);
  m.evl = take((size_t)3 * g.wpc * 32 * 4);
  m.misc = take(64);
  m.total = o;
  return m;
}

// Payload of one evicted slab slot into the cold ring + its index vector, one warp.
template <int DT, int D>
__device__ void step_evict_one(const hc_layer& L, const hc_seq_desc& d, int slot, int dst, int64_t posv) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int PER = (D + 31) / 32;
  const int lane = threadIdx.x & 31;
  if (slot < 0 || slot >= d.cap || dst >= d.ccap) {
    if (lane == 0) set_status(d.st, HC_DEV_INDEX);
    return;
  }
  float mean[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) mean[i] = 0.f;
  T* __restrict__ ck = reinterpret_cast<T*>(d.cold_kpre) + (size_t)dst * L.Hk * D;
  T* __restrict__ cv = reinterpret_cast<T*>(d.cold_v) + (size_t)dst * L.Hk * D;
  for (int h0 = 0; h0 < L.Hk; h0 += 8) {
    const int nh = min(8, L.Hk - h0);
    T kr[8][PER], vr[8][PER];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nh) break;
      const size_t off = ((size_t)(h0 + j) * d.cap + slot) * D;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int dd = lane + 32 * i;
        if (dd < D) {
          kr[j][i] = reinterpret_cast<const T*>(d.hot_kpre)[off + dd];
          vr[j][i] = reinterpret_cast<const T*>(d.hot_v)[off + dd];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nh) break;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int dd = lane + 32 * i;
        if (dd < D) {
          ck[(size_t)(h0 + j) * D + dd] = kr[j][i];
          cv[(size_t)(h0 + j) * D + dd] = vr[j][i];
          mean[i] += E::to_f(kr[j][i]);
        }
      }
    }
  }
  if (lane == 0) d.cold_pos[dst] = posv;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    mean[i] = mean[i] / (float)L.Hk;
    const int dd = lane + 32 * i;
    if (dd < D && dd < L.F) ss += mean[i] * mean[i];
  }
  ss = warp_sum(ss);
  const float den = fmaxf(sqrtf(ss), 1e-12f);
  float* vec = d.cold_vec + (size_t)dst * L.F;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int dd = lane + 32 * i;
    if (dd < D && dd < L.F) vec[dd] = L.normalize ? mean[i] / den : mean[i];
  }
  for (int f = D + lane; f < L.F; f += 32) vec[f] = 0.f;
}

__device__ __forceinline__ Plan step_plan(const hc_layer& L, int budget, int S) {
  Plan p{S, 0, 0, 0, 0};
  if (S <= budget) return p;
  if (L.policy == HC_POLICY_HOTCOLD) {
    const int recent = min(min(L.recent, budget), S);
    const int prefix = S - recent;
    if (prefix <= 0) return p;
    int ntop = (int)((double)budget * L.topk_ratio);
    ntop = max(1, min(ntop, prefix));
    return Plan{S, prefix, ntop, recent, 1};
  }
  const int window = min(L.recent, S);
  const int prefix = S - window;
  return Plan{S, prefix, max(0, min(budget - window, prefix)), window, 1};
}

template <int DT, int D, int G>
__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(StepArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int ESZ = sizeof(T);
  constexpr int KCH = D * ESZ / 16;  // 16-byte chunks per K row; chunk c of row i sits at c ^ (i & 7)
  constexpr int VE = 16 / ESZ;       // elements per chunk
  constexpr int QSTR = D + 8;        // padded row of the MMA query operand (no bank conflicts)
  constexpr int H = D / 2;
  constexpr int RP = ((G + 1) * H + kStepThreads - 1) / kStepThreads;  // RoPE pairs per thread
  static_assert(KCH >= 8, "the chunk swizzle needs rows of at least 128 bytes");
  cg::cluster_group cluster = cg::this_cluster();
  const hc_layer& L = a.L;
  const StepGeom& gm = a.g;
  const int rank = (int)cluster.block_rank();
  const int P = gm.P, ncta = L.Hk * P;
  const int h = rank / P, p = rank % P;
  const int s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tmax = gm.tmax, dpc = gm.dpc;

  // arrival: this CTA has started; waited on before the first distributed shared memory store
  cluster_arrive_relaxed();

  extern __shared__ __align__(128) unsigned char smem[];
  const StepSmem M = step_smem(D, ESZ, G, L.Hk, gm);
  T* sK = reinterpret_cast<T*>(smem + M.k);
  T* sV = reinterpret_cast<T*>(smem + M.v);
  T* sQh = reinterpret_cast<T*>(smem + M.qh);
  float* sQ = reinterpret_cast<float*>(smem + M.q);
  float* sA = reinterpret_cast<float*>(smem + M.a);
  int* sOrd = reinterpret_cast<int*>(smem + M.ord);
  int* sFree = reinterpret_cast<int*>(smem + M.fre);
  int* sHeld = reinterpret_cast<int*>(smem + M.held);
  float* sE = reinterpret_cast<float*>(smem + M.e);
  float* sPool = reinterpret_cast<float*>(smem + M.pool);
  unsigned long long* sBest = reinterpret_cast<unsigned long long*>(smem + M.best);
  uint32_t* sKey = reinterpret_cast<uint32_t*>(smem + M.key);
  float* sRed = reinterpret_cast<float*>(smem + M.red);  // per-warp partials and per-head statistics
  unsigned long long* sRed64 = reinterpret_cast<unsigned long long*>(smem + M.red);
  uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + M.mask);
  int* sCnt = reinterpret_cast<int*>(smem + M.cnt);
  uint32_t* sWord = reinterpret_cast<uint32_t*>(smem + M.word);
  int* sFlag = reinterpret_cast<int*>(smem + M.flag);
  int* sEvl = reinterpret_cast<int*>(smem + M.evl);
  int* sMisc = reinterpret_cast<int*>(smem + M.misc);

  // the descriptor is written once when the layer is set up, so it is read before the wait
  const hc_seq_desc d = L.desc[s];
  pdl_wait();

  // ---- one round trip: counters, logical order, free stack, held flags, new token inputs ----
  hc_seq_state* st = d.st;
  const int n_hot = st->n_hot, n_free = st->n_free, held_len = st->held_len;
  const int qwin_head = st->qwin_head, cold_head = st->cold_head, cold_count = st->cold_count;
  const int64_t cur_pos = a.pos[s];
  const int cap = d.cap;
  const T* __restrict__ qp = reinterpret_cast<const T*>(a.q_pre) + (size_t)s * a.qss;
  const T* __restrict__ kp = reinterpret_cast<const T*>(a.k_pre) + (size_t)s * a.kvss + (size_t)h * D;
  const T* __restrict__ vp = reinterpret_cast<const T*>(a.v) + (size_t)s * a.kvss + (size_t)h * D;
  float rx[RP][2], rc[RP][2], rs[RP][2];
#pragma unroll
  for (int j = 0; j < RP; ++j) {
    const int k = tid + j * kStepThreads;
    if (k < (G + 1) * H) {
      const int g = k / H, i = k % H;
      const T* x = g < G ? qp + (size_t)(h * G + g) * D : kp;
      rx[j][0] = E::to_f(x[i]);
      rx[j][1] = E::to_f(x[i + H]);
      if (a.cos) {
        const T* cs = reinterpret_cast<const T*>(a.cos) + (size_t)s * D;
        const T* sn = reinterpret_cast<const T*>(a.sin) + (size_t)s * D;
        rc[j][0] = E::to_f(cs[i]);
        rc[j][1] = E::to_f(cs[i + H]);
        rs[j][0] = E::to_f(sn[i]);
        rs[j][1] = E::to_f(sn[i + H]);
      } else {
        rc[j][0] = L.inv_freq[i];
      }
    }
  }
  const T vnew = tid < dpc ? vp[p * dpc + tid] : E::from_f(0.f);
  // all loads first, then the stores: one round trip for up to kPre entries per thread
  constexpr int kPre = 4;
  int ov[kPre], fv[kPre];
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int i = tid + j * kStepThreads;
    if (i < cap) {
      ov[j] = d.hot_ord[i];
      fv[j] = d.hot_free[i];
    }
  }
  const int t_h = tid;
  const bool hv_ok = a.use_held && t_h < d.r_max;
  const uint8_t hval = hv_ok ? d.held_valid[t_h] : 0;
  const int64_t hpos = hv_ok ? d.held_pos[t_h] : 0;
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int i = tid + j * kStepThreads;
    if (i < cap) {
      sOrd[i] = ov[j];
      sFree[i] = fv[j];
    }
  }
  for (int i = tid + kPre * kStepThreads; i < cap; i += kStepThreads) {
    sOrd[i] = d.hot_ord[i];
    sFree[i] = d.hot_free[i];
  }
  if (hv_ok) sHeld[t_h] = hval != 0 && hpos <= cur_pos;
  if (a.use_held)
    for (int t = tid + kStepThreads; t < d.r_max; t += kStepThreads)
      sHeld[t] = d.held_valid[t] != 0 && d.held_pos[t] <= cur_pos;
  if (tid == 0) {
    sMisc[2] = 0;
    sMisc[3] = 0;
    sMisc[4] = 0;
  }
  __syncthreads();

  const int n_held = a.use_held ? max(0, min(held_len, d.r_max)) : 0;
  const int new_slot = (n_free > 0 && n_free <= cap) ? sFree[n_free - 1] : -1;
  const int S = n_hot + 1;  // hot tokens after the append (logical index n_hot is the new one)
  const int T_all = n_held + S;
  // every CTA reads the same counters (nothing writes them before barrier 1): a uniform exit
  if (n_hot < 0 || S > cap || S > gm.s_cap || T_all > tmax || new_slot < 0 || new_slot >= cap) {
    if (rank == 0 && tid == 0) set_status(st, HC_DEV_CAPACITY);
    cluster_wait();
    return;
  }
  const Plan pl = step_plan(L, d.budget, S);
  const int n_ev_plan = pl.active ? pl.prefix - pl.ntop : 0;
  const int chunk = (((T_all + P - 1) / P) + 7) & ~7;
  const int t0 = min(p * chunk, T_all);
  int ntl = max(0, min(chunk, T_all - t0));
  if (ntl > gm.tpc) {  // host sizing rules this out
    if (tid == 0) set_status(st, HC_DEV_CAPACITY);
    ntl = gm.tpc;
  }
  const int new_t = n_held + n_hot;
  const int nwords = (S + 31) >> 5;
  // CTA r owns the 32-token words w with w * ncta / nwords == r
  const int w0 = (rank * nwords + ncta - 1) / ncta, w1 = ((rank + 1) * nwords + ncta - 1) / ncta;
  const int own0 = w0 * 32, own_n = max(0, min(w1 * 32, S) - own0), nw_own = w1 - w0;
  const int qwin_slot = d.p_max > 0 ? ((qwin_head % d.p_max) + d.p_max) % d.p_max : 0;
  auto phys_of = [&](int li) { return li < n_hot ? sOrd[li] : new_slot; };

  // ---- gathers: K rows of this CTA's tokens, V columns of every token ---------------------
  // 8 lanes per row, so each warp-wide copy covers whole 128-byte lines of 4 rows
  const T* hk = reinterpret_cast<const T*>(d.hot_k);
  const T* hv = reinterpret_cast<const T*>(d.hot_v);
  const T* gk = reinterpret_cast<const T*>(d.held_k);
  const T* gv = reinterpret_cast<const T*>(d.held_v);
  const int sub8 = tid & 7, rg = tid >> 3;
  for (int i = rg; i < ntl; i += kStepThreads / 8) {
    const int t = t0 + i;
    if (t == new_t) continue;
    const T* src = hk;
    int nb = 16;
    if (t < n_held) {
      src = gk + ((size_t)h * d.r_max + t) * D;
    } else {
      const int slot = sOrd[t - n_held];
      if (slot >= 0 && slot < cap) src = hk + ((size_t)h * cap + slot) * D;
      else nb = 0;  // zero-filled; the token is masked
    }
#pragma unroll
    for (int j = 0; j < KCH / 8; ++j) {
      const int c = j * 8 + sub8;
      cp_async16(sK + (size_t)i * D + (size_t)((c ^ (i & 7)) * VE), nb ? src + c * VE : src, nb);
    }
  }
  cp_async_commit();
  const int vch = dpc / VE, vsh = __ffs(vch) - 1;
  const int lpr = vch < 8 ? vch : 8, lsh = __ffs(lpr) - 1;  // lanes per V row
  for (int k = tid; k < (T_all << lsh); k += kStepThreads) {
    const int t = k >> lsh, l0 = k & (lpr - 1);
    if (t == new_t) continue;
    const T* src = hv;
    int nb = 16;
    if (t < n_held) {
      src = gv + ((size_t)h * d.r_max + t) * D + p * dpc;
    } else {
      const int slot = sOrd[t - n_held];
      if (slot >= 0 && slot < cap) src = hv + ((size_t)h * cap + slot) * D + p * dpc;
      else nb = 0;
    }
    for (int c = l0; c < vch; c += lpr) cp_async16(sV + (size_t)t * dpc + c * VE, nb ? src + c * VE : src, nb);
  }
  cp_async_commit();

  // ---- RoPE of the new token (patch.py:161-162), while the gathers are in flight -----------
  const int new_i = (new_t >= t0 && new_t < t0 + ntl) ? new_t - t0 : -1;
#pragma unroll
  for (int j = 0; j < RP; ++j) {
    const int k = tid + j * kStepThreads;
    if (k >= (G + 1) * H) continue;
    const int g = k / H, i = k % H;
    if (g == G && new_i < 0) continue;
    float c0, s0, c1, s1;
    if (a.cos) {
      c0 = rc[j][0]; c1 = rc[j][1]; s0 = rs[j][0]; s1 = rs[j][1];
    } else {
      rope_cs<DT>(rc[j][0], cur_pos, L.rope_scaling, c0, s0);
      c1 = c0;
      s1 = s0;
    }
    // out[i] = x[i] c - x[i+H] s, out[i+H] = x[i+H] c + x[i] s, rounded like the model's ops
    const float o0 = rope_elem<DT>(rx[j][0], -rx[j][1], c0, s0);
    const float o1 = rope_elem<DT>(rx[j][1], rx[j][0], c1, s1);
    if (g < G) {
      sQ[g * D + i] = E::round(o0);
      sQ[g * D + i + H] = E::round(o1);
      sQh[g * QSTR + i] = E::from_f(o0);
      sQh[g * QSTR + i + H] = E::from_f(o1);
    } else {
      const T k0 = E::from_f(o0), k1 = E::from_f(o1);
      sK[(size_t)new_i * D + (((i / VE) ^ (new_i & 7)) * VE) + i % VE] = k0;
      sK[(size_t)new_i * D + ((((i + H) / VE) ^ (new_i & 7)) * VE) + (i + H) % VE] = k1;
      // the owner of the new token writes its slab rows for head h (cache.py:145-148)
      const size_t off = ((size_t)h * cap + new_slot) * D + i;
      reinterpret_cast<T*>(d.hot_k)[off] = k0;
      reinterpret_cast<T*>(d.hot_k)[off + H] = k1;
      reinterpret_cast<T*>(d.hot_kpre)[off] = E::from_f(rx[j][0]);
      reinterpret_cast<T*>(d.hot_kpre)[off + H] = E::from_f(rx[j][1]);
    }
  }
  if (new_i >= 0)
    for (int i = tid; i < D; i += kStepThreads)
      reinterpret_cast<T*>(d.hot_v)[((size_t)h * cap + new_slot) * D + i] = vp[i];
  if (tid < dpc) sV[(size_t)new_t * dpc + tid] = vnew;
  for (int i = tid; i < (15 - G) * QSTR; i += kStepThreads) sQh[(G + 1) * QSTR + i] = E::from_f(0.f);
  __syncthreads();
  // GQA-mean query of this KV head, rounded to the dtype (cache.py:60-64 / scoring.py:17-26)
  for (int dd = tid; dd < D; dd += kStepThreads) {
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g) acc += sQ[g * D + dd];
    const float qb = E::round(acc / (float)G);
    sQ[G * D + dd] = qb;
    sQh[G * QSTR + dd] = E::from_f(qb);
  }
  cp_async_wait<1>();
  __syncthreads();

  // ---- scoring: G attention logits + the eviction logit per token --------------------------
  auto put = [&](int i, int g, float v) {
    if (i >= ntl || g > G) return;
    const int t = t0 + i;
    if (g < G) {
      bool valid = true;
      if (t < n_held) {
        valid = sHeld[t] != 0;
      } else if (t != new_t) {
        const int slot = sOrd[t - n_held];
        valid = slot >= 0 && slot < cap;
        if (!valid && g == 0) set_status(st, HC_DEV_INDEX);
      }
      sA[g * tmax + t] = valid ? v * L.scale : kNegInf;
    } else {
      sE[t] = v;
    }
  };
  if constexpr (DT != HC_F32) {
    const int gid = lane >> 2, tig = lane & 3;
    uint32_t af[D / 16][4];
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int kk = ks * 16 + 2 * tig;
      af[ks][0] = *reinterpret_cast<const uint32_t*>(sQh + gid * QSTR + kk);
      af[ks][1] = *reinterpret_cast<const uint32_t*>(sQh + (gid + 8) * QSTR + kk);
      af[ks][2] = *reinterpret_cast<const uint32_t*>(sQh + gid * QSTR + kk + 8);
      af[ks][3] = *reinterpret_cast<const uint32_t*>(sQh + (gid + 8) * QSTR + kk + 8);
    }
    const int ntiles = (ntl + 7) >> 3;
    const int mat = lane >> 3, r8 = lane & 7;
    // two independent tiles per pass keep two MMA chains in flight
    for (int nt = warp; nt < ntiles; nt += 2 * kStepWarps) {
      const bool two = nt + kStepWarps < ntiles;  // warp-uniform
      const T* row0 = sK + (size_t)(nt * 8 + r8) * D;
      const T* row1 = sK + (size_t)((nt + kStepWarps) * 8 + r8) * D;
      float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kq = 0; kq < D / 32; ++kq) {
        const int ch = ((kq * 4 + mat) ^ r8) * VE;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(row0 + ch, b0, b1, b2, b3);
        mma16816<DT>(c0, af[2 * kq], b0, b1);
        mma16816<DT>(c0, af[2 * kq + 1], b2, b3);
        if (two) {
          ldsm_x4(row1 + ch, b0, b1, b2, b3);
          mma16816<DT>(c1, af[2 * kq], b0, b1);
          mma16816<DT>(c1, af[2 * kq + 1], b2, b3);
        }
      }
      const int n0 = nt * 8 + 2 * tig;
      put(n0, gid, c0[0]);
      put(n0 + 1, gid, c0[1]);
      put(n0, gid + 8, c0[2]);
      put(n0 + 1, gid + 8, c0[3]);
      if (two) {
        const int n1 = n0 + kStepWarps * 8;
        put(n1, gid, c1[0]);
        put(n1 + 1, gid, c1[1]);
        put(n1, gid + 8, c1[2]);
        put(n1 + 1, gid + 8, c1[3]);
      }
    }
  } else {
    const int sub = lane & 7, tk = lane >> 3;
    for (int base = warp * 4; base < ntl; base += 4 * kStepWarps) {
      const int i = base + tk;
      float acc[G + 1];
#pragma unroll
      for (int g = 0; g <= G; ++g) acc[g] = 0.f;
      if (i < ntl) {
        const T* row = sK + (size_t)i * D;
#pragma unroll
        for (int j = 0; j < KCH / 8; ++j) {
          const int c = j * 8 + sub;
          const float4 kv = *reinterpret_cast<const float4*>(row + ((c ^ (i & 7)) * VE));
#pragma unroll
          for (int g = 0; g <= G; ++g) {
            const float4 q = *reinterpret_cast<const float4*>(sQ + g * D + c * VE);
            acc[g] = fmaf(q.x, kv.x, acc[g]);
            acc[g] = fmaf(q.y, kv.y, acc[g]);
            acc[g] = fmaf(q.z, kv.z, acc[g]);
            acc[g] = fmaf(q.w, kv.w, acc[g]);
          }
        }
      }
#pragma unroll
      for (int g = 0; g <= G; ++g) {
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 4);
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
        acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
      }
      if (sub == 0)
#pragma unroll
        for (int g = 0; g <= G; ++g) put(i, g, acc[g]);
    }
  }
  __syncthreads();

  // ---- exchange within head h: attention logits and the eviction row ------------------------
  // Rows are copied as 16-byte vectors: t0 and tmax are multiples of 8, and the up to 3
  // floats past this CTA's tokens land on positions no CTA owns.
  const bool policy = pl.active && n_ev_plan > 0;
  cluster_wait();  // every CTA of the cluster has started
  const int n4 = (ntl + 3) >> 2;
  if (P > 1 && n4 > 0) {
    const int rows = G + (policy ? 1 : 0);
    const int n = rows * n4;
    for (int k = tid; k < (P - 1) * n; k += kStepThreads) {
      const int j = k / n, r = k - j * n, g = r / n4, i = r - g * n4;
      float* base = g < G ? sA + (size_t)g * tmax : sE;
      const size_t idx = (size_t)t0 + 4 * i;
      *reinterpret_cast<float4*>(cluster.map_shared_rank(base, h * P + (j < p ? j : j + 1)) + idx) =
          *reinterpret_cast<const float4*>(base + idx);
    }
  }
  cluster.sync();

  // ---- policy: per-head values pooled by the CTAs of each head, summed by token owners ------
  int n_ev = 0;
  if (policy) {
    const int wpc32 = gm.wpc * 32;
    float* x = sE + n_held;  // eviction logit of logical index li of head h
    const int pb = p * pl.prefix / P, pe = (p + 1) * pl.prefix / P;  // this CTA's share of the prefix
    auto send = [&](int li, float v) {
      const int w = li >> 5;
      const int r2 = w * ncta / nwords;
      const int o0 = ((r2 * nwords + ncta - 1) / ncta) * 32;
      cluster.map_shared_rank(sPool, r2)[h * wpc32 + (li - o0)] = v;
    };
    if (L.policy == HC_POLICY_SNAPKV) {
      // softmax over every hot token of head h (the single observation row sees every key)
      float m = kNegInf;
      for (int li = tid; li < S; li += kStepThreads) m = fmaxf(m, x[li] * L.scale);
      m = warp_max(m);
      if (lane == 0) sRed[warp] = m;
      __syncthreads();
      m = sRed[0];
#pragma unroll
      for (int w = 1; w < kStepWarps; ++w) m = fmaxf(m, sRed[w]);
      float l = 0.f;
      for (int li = tid; li < S; li += kStepThreads) {
        const float e = __expf(x[li] * L.scale - m);
        x[li] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) sRed[kStepWarps + warp] = l;
      __syncthreads();
      l = 0.f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) l += sRed[kStepWarps + w];
      const int pad = L.pool_kernel > 1 ? L.pool_kernel / 2 : 0;
      const bool pmax = L.pooling == HC_POOL_MAX;
      for (int li = pb + tid; li < pe; li += kStepThreads) {
        float v;
        if (pad == 0) {
          v = x[li] / l;
        } else if (pmax) {
          // max of e/l over the window equals (max e)/l: the division is monotone
          v = kNegInf;
          if (pad <= 7) {
#pragma unroll
            for (int o = -7; o <= 7; ++o) {
              const int u = li + o;
              if (o >= -pad && o <= pad && u >= 0 && u < S) v = fmaxf(v, x[u]);
            }
          } else {
            for (int u = max(0, li - pad); u <= min(S - 1, li + pad); ++u) v = fmaxf(v, x[u]);
          }
          v = v / l;
        } else {
          v = 0.f;
          for (int u = max(0, li - pad); u <= min(S - 1, li + pad); ++u) v += x[u] / l;
          v /= (float)L.pool_kernel;
        }
        send(li, v);
      }
    } else {
      for (int li = pb + tid; li < pe; li += kStepThreads) send(li, x[li]);
    }
    cluster.sync();

    // token owners: mean over heads (cache.py:60-64 hot/cold sum; SnapKV head mean)
    const float inv = 1.f / sqrtf((float)L.D);
    const bool snap = L.policy == HC_POLICY_SNAPKV;
    unsigned long long best = ~0ull;
    for (int i = tid; i < own_n; i += kStepThreads) {
      const int li = own0 + i;
      if (li >= pl.prefix) break;
      float tot = 0.f;
      for (int hh = 0; hh < L.Hk; ++hh) tot += snap ? sPool[hh * wpc32 + i] : sPool[hh * wpc32 + i] * inv;
      const uint32_t key = fkey(tot / (float)L.Hk);
      sKey[li] = key;
      const unsigned long long c = ((unsigned long long)key << 32) | (0xffffffffu - (uint32_t)li);
      best = c < best ? c : best;
    }
    n_ev = n_ev_plan;
    if (n_ev == 1) {
      // one token leaves: the lowest key, equal keys evict the higher index
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
        best = y < best ? y : best;
      }
      if (lane == 0) sRed64[warp] = best;
      __syncthreads();
      if (tid < ncta) {
        unsigned long long b = sRed64[0];
#pragma unroll
        for (int w = 1; w < kStepWarps; ++w) b = sRed64[w] < b ? sRed64[w] : b;
        cluster.map_shared_rank(sBest, tid)[rank] = b;
      }
      cluster.sync();
      best = sBest[0];
      for (int r2 = 1; r2 < ncta; ++r2) best = sBest[r2] < best ? sBest[r2] : best;
      const int li_ev = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
      // compaction of own words: entries after li_ev move down by one
      for (int i = tid; i < own_n; i += kStepThreads) {
        const int li = own0 + i;
        const int ph = phys_of(li);
        if (li > li_ev) {
          d.hot_ord[li - 1] = ph;
        } else if (li == li_ev) {
          if (n_free - 1 < cap) d.hot_free[n_free - 1] = ph;
          sEvl[0] = ph;
          sEvl[1] = d.ccap > 0 ? (int)(((long)cold_head + cold_count) % d.ccap) : -1;
          sEvl[2] = li;
          sMisc[4] = 1;
        }
      }
      if (tid < G) sA[tid * tmax + n_held + li_ev] = kNegInf;
      __syncthreads();
    } else {
      // keys of own tokens to every CTA, then the rank of each own token among the prefix
      __syncthreads();
      for (int k = tid; k < ncta * own_n; k += kStepThreads) {
        const int r2 = k / own_n, i = k - r2 * own_n, li = own0 + i;
        if (li < pl.prefix && r2 != rank) cluster.map_shared_rank(sKey, r2)[li] = sKey[li];
      }
      cluster.sync();
      int tpt = kStepThreads / (gm.wpc * 32);
      tpt = tpt >= 32 ? 32 : tpt >= 16 ? 16 : tpt >= 8 ? 8 : tpt >= 4 ? 4 : tpt >= 2 ? 2 : 1;
      const int tsh = __ffs(tpt) - 1;
      for (int base = 0; base < own_n * tpt; base += kStepThreads) {
        const int k = base + tid, tl = k >> tsh, sub = k & (tpt - 1), t = own0 + tl;
        int cnt = 0;
        if (tl < own_n && t < pl.prefix) {
          const uint32_t kt = sKey[t];
#pragma unroll 4
          for (int u = sub; u < pl.prefix; u += tpt) {
            const uint32_t ku = sKey[u];
            cnt += (ku > kt) || (ku == kt && u < t);
          }
        }
        for (int o = 1; o < tpt; o <<= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
        if (sub == 0 && tl < own_n) sFlag[tl] = (t >= pl.prefix) || (cnt < pl.ntop);
      }
      __syncthreads();
      for (int wi = warp; wi < nw_own; wi += kStepWarps) {
        const int t = own0 + wi * 32 + lane;
        const bool in = t < S;
        const bool keep = in && sFlag[wi * 32 + lane];
        const unsigned evw = __ballot_sync(0xffffffffu, in && !keep);
        const unsigned kpw = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) {
          sWord[wi] = evw;
          atomicAdd(&sMisc[2], __popc(kpw));
          atomicAdd(&sMisc[3], __popc(evw));
        }
      }
      __syncthreads();
      const int nb = nw_own + 2;
      for (int k = tid; k < ncta * nb; k += kStepThreads) {
        const int r2 = k / nb, j = k - r2 * nb;
        if (j < nw_own) cluster.map_shared_rank(sMask, r2)[w0 + j] = sWord[j];
        else cluster.map_shared_rank(sCnt, r2)[2 * rank + (j - nw_own)] = sMisc[2 + j - nw_own];
      }
      cluster.sync();

      int kb = 0, eb = 0, tot_ev = 0;
      for (int r2 = 0; r2 < ncta; ++r2) {
        const int kc = sCnt[2 * r2], ec = sCnt[2 * r2 + 1];
        tot_ev += ec;
        if (r2 < rank) {
          kb += kc;
          eb += ec;
        }
      }
      n_ev = tot_ev;
      // compaction of own words: new logical order, freed slots, cold-ring destinations
      if (warp == 0) {
        int nloc = 0;
        const unsigned lt = (1u << lane) - 1u;
        for (int wi = 0; wi < nw_own; ++wi) {
          const int t = own0 + wi * 32 + lane;
          const bool in = t < S;
          const bool ev = in && ((sMask[w0 + wi] >> lane) & 1u);
          const bool keep = in && !ev;
          const unsigned km = __ballot_sync(0xffffffffu, keep), em = __ballot_sync(0xffffffffu, ev);
          const int ph = in ? phys_of(t) : -1;
          if (keep) d.hot_ord[kb + __popc(km & lt)] = ph;
          if (ev) {
            const int j = eb + __popc(em & lt), jl = nloc + __popc(em & lt);
            if (n_free - 1 + j < cap) d.hot_free[n_free - 1 + j] = ph;
            sEvl[3 * jl] = ph;
            sEvl[3 * jl + 1] = (j >= n_ev - d.ccap) ? (int)(((long)cold_head + cold_count + j) % d.ccap) : -1;
            sEvl[3 * jl + 2] = t;
          }
          kb += __popc(km);
          eb += __popc(em);
          nloc += __popc(em);
        }
        if (lane == 0) sMisc[4] = nloc;
      }
      for (int li = tid; li < S; li += kStepThreads)
        if ((sMask[li >> 5] >> (li & 31)) & 1u)
#pragma unroll
          for (int g = 0; g < G; ++g) sA[g * tmax + n_held + li] = kNegInf;
      __syncthreads();
    }
  }

  // ---- softmax over every token of head h, P.V for this CTA's columns ----------------------
  float* sPm = sRed + 4 * kStepMaxCluster;
  {
    constexpr int WPG = kStepWarps / G;
    const int g = warp % G, sl = warp / G;
    float m = kNegInf;
    for (int t = sl * 32 + lane; t < T_all; t += WPG * 32) m = fmaxf(m, sA[g * tmax + t]);
    m = warp_max(m);
    if (lane == 0) sPm[warp] = m;
  }
  __syncthreads();
  float mg[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float m = kNegInf;
    for (int sl = 0; sl < kStepWarps / G; ++sl) m = fmaxf(m, sPm[sl * G + g]);
    mg[g] = m;
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
    for (int t = tid; t < T_all; t += kStepThreads) {
      const float x = sA[g * tmax + t];
      sA[g * tmax + t] = (x == kNegInf) ? 0.f : __expf(x - mg[g]);
    }
  cp_async_wait<0>();
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem + M.k);  // the K rows are no longer needed
  float* redl = red + (size_t)kStepWarps * G * dpc;
  {
    const int c = tid & (vch - 1), grp = tid >> vsh, ngrp = kStepThreads >> vsh;
    float o[G][VE], l[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      l[g] = 0.f;
#pragma unroll
      for (int e = 0; e < VE; ++e) o[g][e] = 0.f;
    }
    for (int t = grp; t < T_all; t += ngrp) {
      float vf[VE];
      unpack16<DT>(*reinterpret_cast<const uint4*>(sV + (size_t)t * dpc + c * VE), vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = sA[g * tmax + t];
        l[g] += pr;
#pragma unroll
        for (int e = 0; e < VE; ++e) o[g][e] = fmaf(pr, vf[e], o[g][e]);
      }
    }
    for (int off = vch; off < 32; off <<= 1) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
#pragma unroll
        for (int e = 0; e < VE; ++e) o[g][e] += __shfl_xor_sync(0xffffffffu, o[g][e], off);
      }
    }
    if (lane < vch) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int e = 0; e < VE; ++e) red[((size_t)warp * G + g) * dpc + c * VE + e] = o[g][e];
        if (c == 0) redl[warp * G + g] = l[g];
      }
    }
  }
  __syncthreads();
  T* outp = reinterpret_cast<T*>(a.out) + ((size_t)s * L.Hq + (size_t)h * G) * D + (size_t)p * dpc;
#pragma unroll
  for (int g = 0; g < G; ++g)
    for (int dd = tid; dd < dpc; dd += kStepThreads) {
      float os = 0.f, ls = 0.f;
#pragma unroll 4
      for (int w = 0; w < kStepWarps; ++w) {
        os += red[((size_t)w * G + g) * dpc + dd];
        ls += redl[w * G + g];
      }
      float r = os / ls;
      if (a.overflow_nan && mg[g] >= kExpOverflow) r = __int_as_float(0x7fc00000);
      outp[(size_t)g * D + dd] = E::from_f(r);
    }

  // ---- counters (one thread of CTA 0) --------------------------------------------------------
  if (rank == 0 && tid == 0) {
    d.hot_pos[new_slot] = cur_pos;
    if (n_ev == 0) d.hot_ord[n_hot] = new_slot;
    if (n_ev > 0) {
      const long total = (long)cold_count + n_ev;
      if (total > d.ccap) {
        st->cold_head = (int)(((long)cold_head + total - d.ccap) % d.ccap);
        st->cold_count = d.ccap;
      } else {
        st->cold_count = (int)total;
      }
    }
    st->n_evict = n_ev;
    st->n_hot = S - n_ev;
    st->n_free = n_free - 1 + n_ev;
    if (d.p_max > 0) st->qwin_head = (qwin_slot + 1) % d.p_max;
  }
  // ---- work nothing in this kernel waits for: evicted payloads, query pool -------------------
  if (n_ev > 0) {
    const int nloc = sMisc[4];
    for (int q = warp; q < nloc; q += kStepWarps) {
      const int slot = sEvl[3 * q], dst = sEvl[3 * q + 1], li = sEvl[3 * q + 2];
      if (dst < 0) continue;  // more tokens evicted than the ring holds: the oldest are dropped
      const int64_t pv = li == n_hot ? cur_pos : (slot >= 0 && slot < cap ? d.hot_pos[slot] : -1);
      step_evict_one<DT, D>(L, d, slot, dst, pv);
    }
  }
  // query pool push: mean over all query heads of the pre-RoPE query (controller.py:240-241)
  if (rank == ncta - 1 && d.p_max > 0) {
    for (int dd = tid; dd < D; dd += kStepThreads) {
      float acc = 0.f;
#pragma unroll 8
      for (int hh = 0; hh < L.Hq; ++hh) acc += E::to_f(qp[(size_t)hh * D + dd]);
      reinterpret_cast<T*>(d.qwin)[(size_t)qwin_slot * D + dd] = E::from_f(acc / (float)L.Hq);
    }
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
int step_parts(int Hk) { return (Hk >= 1 && Hk <= kStepMaxCluster && kStepMaxCluster % Hk == 0) ? kStepMaxCluster / Hk : 0; }

static StepGeom layer_geom(const hc_layer& L, int use_held) {
  return step_geom(L.Hk, L.D, L.max_cap, L.max_r, use_held);
}

size_t step_smem_bytes(const hc_layer& L, int use_held) {
  const StepGeom g = layer_geom(L, use_held);
  if (!g.P || L.Hq % L.Hk) return 0;
  const int esz = L.dtype == HC_F32 ? 4 : 2;
  const int G = L.Hq / L.Hk;
  if (G > 8 || g.dpc * esz < 16 || (g.dpc * esz) % 16 || (L.D * esz) < 128) return 0;
  return step_smem(L.D, esz, G, L.Hk, g).total;
}

// Per-(kernel, shared memory size) launch checks, done once: the cluster-size opt-in and
// whether one 16-CTA cluster of this size is schedulable on the device.
template <typename K>
static cudaError_t step_prepare(K kern, cudaLaunchConfig_t* cfg) {
  struct Entry {
    const void* fn;
    int dev;
    size_t bytes;
    int ok;
  };
  static Entry cache[64];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const void* fn = reinterpret_cast<const void*>(kern);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i)
      if (cache[i].fn == fn && cache[i].dev == dev && cache[i].bytes == cfg->dynamicSmemBytes)
        return cache[i].ok ? cudaSuccess : cudaErrorNotSupported;
  }
  e = ensure_smem(kern, cfg->dynamicSmemBytes);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, kern, cfg);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (n < 64) cache[n++] = Entry{fn, dev, cfg->dynamicSmemBytes, clusters >= 1};
  return clusters >= 1 ? cudaSuccess : cudaErrorNotSupported;
}

template <int DT, int D, int G>
static cudaError_t step_t(const StepArgs& a, cudaStream_t stream) {
  using T = typename Elem<DT>::T;
  const StepSmem M = step_smem(D, sizeof(T), G, a.L.Hk, a.g);
  auto kern = step_kernel<DT, D, G>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.L.Hk * a.g.P, a.L.n_seq);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = M.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.L.Hk * a.g.P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = step_prepare(kern, &cfg);
  if (e != cudaSuccess) return e;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int DT, int D>
static cudaError_t step_g(const StepArgs& a, cudaStream_t stream) {
  switch (a.L.Hq / a.L.Hk) {
    case 1: return step_t<DT, D, 1>(a, stream);
    case 2: return step_t<DT, D, 2>(a, stream);
    case 4: return step_t<DT, D, 4>(a, stream);
    case 8: return step_t<DT, D, 8>(a, stream);
  }
  return cudaErrorNotSupported;
}

cudaError_t launch_step(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                        const void* c, const void* sn, const int64_t* pos, int use_held, void* out, int overflow_nan,
                        cudaStream_t stream) {
  if (!step_smem_bytes(L, use_held)) return cudaErrorNotSupported;
  StepArgs a{};
  a.L = L;
  a.q_pre = q;
  a.qss = qss;
  a.k_pre = k;
  a.v = v;
  a.kvss = kvss;
  a.cos = c;
  a.sin = sn;
  a.pos = pos;
  a.out = out;
  a.use_held = use_held;
  a.overflow_nan = overflow_nan;
  a.g = layer_geom(L, use_held);
  if (L.dtype == HC_F32 && L.D == 128) return step_g<HC_F32, 128>(a, stream);
  if (L.dtype == HC_F16 && L.D == 128) return step_g<HC_F16, 128>(a, stream);
  if (L.dtype == HC_BF16 && L.D == 128) return step_g<HC_BF16, 128>(a, stream);
  if (L.dtype == HC_F32 && L.D == 64) return step_g<HC_F32, 64>(a, stream);
  if (L.dtype == HC_F16 && L.D == 64) return step_g<HC_F16, 64>(a, stream);
  if (L.dtype == HC_BF16 && L.D == 64) return step_g<HC_BF16, 64>(a, stream);
  return cudaErrorNotSupported;
}

}  // namespace hc
