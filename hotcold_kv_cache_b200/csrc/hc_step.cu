// Fused decode step of one layer: append, compression with eviction into the cold ring, and
// attention over [held | hot] in one launch — one thread-block cluster per sequence.
//
// The reference runs this as a chain of torch ops and a Triton kernel per layer
// (patch.py:161-305 with cache.py:130-151 and cache.py:37-128). Split into separate kernels
// (hc_append, hc_compress, hc_attend) the step pays a launch and a global round trip per
// stage; at batch 1 that latency, not HBM bandwidth, sets the time. Here the cluster holds
// Hk*P CTAs, CTA (h, p) owning KV head h and part p of the sequence's token list:
//   1. every CTA bulk-copies the K/V rows of its tokens into shared memory, RoPEs the new
//      token's query heads of its group (and, for the owner of the new token, its key), and
//      scores each token once: G attention logits and the eviction logit (GQA-mean query . k);
//   2. eviction logits go to the leader CTA through distributed shared memory; the leader
//      applies the policy (hot/cold sum, or SnapKV softmax + pooling + head mean), selects the
//      tokens to keep (exact top-k, ties to the lower index) and publishes the evicted set;
//   3. every CTA masks its evicted tokens out of its partial softmax (K/V are still resident),
//      head leaders merge the P partials through distributed shared memory and write the
//      output; the leader compacts the logical order, pushes freed slots, and the CTAs copy
//      evicted payloads into the cold ring with their index vectors.
// The result equals hc_append + hc_compress + hc_attend on the same state.

#include <cooperative_groups.h>

#include "hc_internal.cuh"
#include "hc_topk.cuh"

namespace cg = cooperative_groups;

namespace hc {

constexpr int kStepThreads = 256;
constexpr int kStepMaxCluster = 16;

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
  int P;      // parts per KV head; cluster = Hk * P
  int tpc;    // token rows per CTA
  int s_cap;  // leader arrays: max hot tokens
};

struct StepSmem {
  size_t k, v, q, qbar, sc, info, ml, part, e, tok, sel, evmask, evlist, ord, evcopy, topk, misc, bars, total;
};

__host__ __device__ inline size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline StepSmem step_smem(int D, int esz, int G, int tpc, int s_cap, int P, int Hk) {
  StepSmem m{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t r = o; o += al16(b); return r; };
  m.k = take((size_t)tpc * D * esz);
  m.v = take((size_t)tpc * D * esz);
  m.q = take((size_t)G * D * 4);
  m.qbar = take((size_t)D * 4);
  // attention scores [G][tpc]; after P.V the same area folds the (256/D - 1) extra partial sums
  m.sc = take((size_t)4 * (G * tpc > (kStepThreads / D - 1) * G * D ? G * tpc : (kStepThreads / D - 1) * G * D));
  m.info = take((size_t)3 * tpc * 4);      // logical index / valid / physical slot per row
  m.ml = take((size_t)2 * G * 4);
  m.part = take((size_t)P * (G * D + 2 * G) * 4);
  m.e = take((size_t)Hk * s_cap * 4);      // leader: eviction logits [Hk][S]
  m.tok = take((size_t)Hk * s_cap * 4 + (size_t)s_cap * 4);  // leader: importance [Hk][S] + scores [S]
  m.sel = take((size_t)s_cap);
  m.evmask = take((size_t)((s_cap + 31) / 32) * 4);
  m.evlist = take((size_t)3 * s_cap * 4);  // leader: (slot, ring dst) per evicted token + count
  m.ord = take((size_t)2 * s_cap * 4);     // leader: old logical order, then the new one
  m.evcopy = take((size_t)2 * (s_cap / kStepMaxCluster + 2) * 4);  // this CTA's evicted (slot, dst) pairs
  m.topk = take((size_t)kTopkSmemInts * 4);
  m.misc = take(64);
  m.bars = take(16);
  m.total = o;
  return m;
}

// Payload of one evicted slab slot into the cold ring + its index vector, one warp.
template <int DT, int D>
__device__ void step_evict_one(const hc_layer& L, const hc_seq_desc& d, int slot, int dst) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int PER = (D + 31) / 32;
  const int lane = threadIdx.x & 31;
  if (slot < 0 || slot >= d.cap || dst < 0 || dst >= d.ccap) {
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
  if (lane == 0) d.cold_pos[dst] = d.hot_pos[slot];
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
__global__ void __launch_bounds__(kStepThreads) step_kernel(StepArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int ROWB = D * sizeof(T);
  constexpr int VEC = 16 / sizeof(T);
  constexpr int NJ = D / (8 * VEC);
  constexpr int H = D / 2;
  cg::cluster_group cluster = cg::this_cluster();
  const hc_layer& L = a.L;
  const int rank = (int)cluster.block_rank();
  const int h = rank / a.P, p = rank % a.P;
  const int s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  extern __shared__ __align__(128) unsigned char smem[];
  const StepSmem M = step_smem(D, sizeof(T), G, a.tpc, a.s_cap, a.P, L.Hk);
  T* sK = reinterpret_cast<T*>(smem + M.k);
  T* sV = reinterpret_cast<T*>(smem + M.v);
  float* sQ = reinterpret_cast<float*>(smem + M.q);
  float* sQbar = reinterpret_cast<float*>(smem + M.qbar);
  float* sS = reinterpret_cast<float*>(smem + M.sc);
  int* sLog = reinterpret_cast<int*>(smem + M.info);
  int* sValid = sLog + a.tpc;
  int* sSlot = sValid + a.tpc;
  float* sML = reinterpret_cast<float*>(smem + M.ml);
  float* sPart = reinterpret_cast<float*>(smem + M.part);
  float* sE = reinterpret_cast<float*>(smem + M.e);
  float* sImp = reinterpret_cast<float*>(smem + M.tok);
  float* sTok = sImp + (size_t)L.Hk * a.s_cap;
  uint8_t* sSel = reinterpret_cast<uint8_t*>(smem + M.sel);
  uint32_t* sEvMask = reinterpret_cast<uint32_t*>(smem + M.evmask);
  int* sEvList = reinterpret_cast<int*>(smem + M.evlist);
  int* sOldOrd = reinterpret_cast<int*>(smem + M.ord);
  int* sOrd = sOldOrd + a.s_cap;
  int* sEvCopy = reinterpret_cast<int*>(smem + M.evcopy);
  int* sTopk = reinterpret_cast<int*>(smem + M.topk);
  int* sMisc = reinterpret_cast<int*>(smem + M.misc);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + M.bars);

  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  hc_seq_state* st = d.st;
  const int n_hot = st->n_hot, n_free = st->n_free;
  const int n_held = a.use_held ? max(0, min(st->held_len, d.r_max)) : 0;
  const int new_slot = (n_free > 0 && n_free <= d.cap) ? d.hot_free[n_free - 1] : -1;
  // the same counters are read by every CTA of the cluster, so this exit is cluster-uniform
  if (n_hot < 0 || n_hot + 1 > d.cap || new_slot < 0 || new_slot >= d.cap) {
    if (rank == 0 && tid == 0) set_status(st, HC_DEV_CAPACITY);
    return;
  }
  const int S = n_hot + 1;  // hot tokens after the append (logical index n_hot is the new one)
  const Plan pl = step_plan(L, d.budget, S);
  const int T_all = n_held + S;
  const int chunk = (T_all + a.P - 1) / a.P;
  const int t0 = p * chunk, nt = max(0, min(chunk, T_all - t0));
  const int64_t cur_pos = a.pos[s];
  const int qwin_slot = d.p_max > 0 ? ((st->qwin_head % d.p_max) + d.p_max) % d.p_max : 0;
  const int ncta = L.Hk * a.P;
  if (nt > a.tpc) {  // host sizing guarantees this never happens; report and keep going safely
    if (tid == 0) set_status(st, HC_DEV_CAPACITY);
  }
  const int ntl = min(nt, a.tpc);

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
    sMisc[1] = 0;
  }
  __syncthreads();
  // ---- rows of this CTA's tokens (a CTA may hold more tokens than it has threads) ----------
  int my_copies = 0;
  for (int i = tid; i < ntl; i += kStepThreads) {
    const int t = t0 + i;
    const T* krow = nullptr;
    const T* vrow = nullptr;
    int logical = -1, valid = 1, slot = -1;
    if (t < n_held) {
      const size_t off = ((size_t)h * d.r_max + t) * D;
      krow = reinterpret_cast<const T*>(d.held_k) + off;
      vrow = reinterpret_cast<const T*>(d.held_v) + off;
      valid = d.held_valid[t] != 0 && d.held_pos[t] <= cur_pos;
    } else {
      logical = t - n_held;
      if (logical < n_hot) {
        slot = d.hot_ord[logical];
        if (slot >= 0 && slot < d.cap) {
          const size_t off = ((size_t)h * d.cap + slot) * D;
          krow = reinterpret_cast<const T*>(d.hot_k) + off;
          vrow = reinterpret_cast<const T*>(d.hot_v) + off;
        } else {
          valid = 0;
          set_status(st, HC_DEV_INDEX);
        }
      } else {
        slot = new_slot;  // the new token: its rows are computed below
      }
    }
    sLog[i] = logical;
    sValid[i] = valid;
    sSlot[i] = slot;
    if (krow) {
      // issued before the expected byte count is posted: the barrier's pending arrival keeps
      // the phase open, and its transaction count may run negative in the meantime
      bulk_g2s(sK + (size_t)i * D, krow, ROWB, &bars[0]);
      bulk_g2s(sV + (size_t)i * D, vrow, ROWB, &bars[1]);
      ++my_copies;
    } else if (logical < 0 || logical < n_hot) {
      for (int e = 0; e < D; ++e) {
        sK[(size_t)i * D + e] = E::from_f(0.f);
        sV[(size_t)i * D + e] = E::from_f(0.f);
      }
    }
  }
  if (my_copies) atomicAdd(&sMisc[1], my_copies);
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], (uint32_t)(sMisc[1] * ROWB));
    mbar_arrive_expect_tx(&bars[1], (uint32_t)(sMisc[1] * ROWB));
  }
  // the leader's copy of the logical order, loaded while the rows are in flight
  if (rank == 0 && pl.active)
    for (int i = tid; i < n_hot; i += kStepThreads) sOldOrd[i] = d.hot_ord[i];
  // ---- RoPE of the new token (patch.py:161-162), while the rows are in flight --------------
  const T* __restrict__ qp = reinterpret_cast<const T*>(a.q_pre) + (size_t)s * a.qss;
  const T* __restrict__ kp = reinterpret_cast<const T*>(a.k_pre) + (size_t)s * a.kvss + (size_t)h * D;
  const T* __restrict__ vp = reinterpret_cast<const T*>(a.v) + (size_t)s * a.kvss + (size_t)h * D;
  const int new_row = (n_held + n_hot >= t0 && n_held + n_hot < t0 + ntl) ? n_held + n_hot - t0 : -1;
  for (int i = tid; i < (G + 1) * D; i += kStepThreads) {
    const int g = i / D, dd = i % D;
    float c, sn;
    if (a.cos) {
      c = E::load(reinterpret_cast<const T*>(a.cos) + (size_t)s * D + dd);
      sn = E::load(reinterpret_cast<const T*>(a.sin) + (size_t)s * D + dd);
    } else {
      rope_cs<DT>(L.inv_freq[dd % H], cur_pos, L.rope_scaling, c, sn);
    }
    if (g < G) {
      const T* x = qp + (size_t)(h * G + g) * D;
      const float r = dd < H ? -E::to_f(x[dd + H]) : E::to_f(x[dd - H]);
      sQ[g * D + dd] = E::round(rope_elem<DT>(E::to_f(x[dd]), r, c, sn));
    } else {
      const float r = dd < H ? -E::to_f(kp[dd + H]) : E::to_f(kp[dd - H]);
      const T kpost = E::from_f(rope_elem<DT>(E::to_f(kp[dd]), r, c, sn));
      if (new_row >= 0) {
        sK[(size_t)new_row * D + dd] = kpost;
        sV[(size_t)new_row * D + dd] = vp[dd];
        // the owner of the new token writes its slab rows for head h (cache.py:145-148)
        const size_t off = ((size_t)h * d.cap + new_slot) * D + dd;
        reinterpret_cast<T*>(d.hot_k)[off] = kpost;
        reinterpret_cast<T*>(d.hot_kpre)[off] = kp[dd];
        reinterpret_cast<T*>(d.hot_v)[off] = vp[dd];
      }
    }
  }
  __syncthreads();
  // GQA-mean query of this KV head, rounded to the dtype (cache.py:60-64 / scoring.py:17-26)
  for (int dd = tid; dd < D; dd += kStepThreads) {
    float acc = 0.f;
    for (int g = 0; g < G; ++g) acc += sQ[g * D + dd];
    sQbar[dd] = E::round(acc / (float)G);
  }
  // every CTA of the cluster is running before any distributed shared memory access
  cluster.sync();

  // ---- one scoring pass: G attention logits + the eviction logit per token ----------------
  const int sub = lane & 7, tk = lane >> 3;
  float qr[G + 1][NJ * VEC];
#pragma unroll
  for (int g = 0; g <= G; ++g)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        qr[g][j * VEC + e] = (g < G ? sQ + g * D : sQbar)[j * 8 * VEC + sub * VEC + e];
  if (!__syncthreads_and(mbar_wait(&bars[0], 0))) {
    if (tid == 0) set_status(st, HC_DEV_TIMEOUT);
    mbar_wait(&bars[1], 0);
  }
  float* leaderE = cluster.map_shared_rank(sE, 0);
  for (int base = warp * 4; base < ntl; base += 4 * (kStepThreads / 32)) {
    const int t = base + tk;
    float acc[G + 1];
#pragma unroll
    for (int g = 0; g <= G; ++g) acc[g] = 0.f;
    if (t < ntl) {
      const T* row = sK + (size_t)t * D;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        uint4 u = *reinterpret_cast<const uint4*>(row + j * 8 * VEC + sub * VEC);
        float kf[VEC];
        unpack16<DT>(u, kf);
#pragma unroll
        for (int g = 0; g <= G; ++g)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[g] = fmaf(qr[g][j * VEC + e], kf[e], acc[g]);
      }
    }
#pragma unroll
    for (int g = 0; g <= G; ++g) {
      acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 4);
      acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 2);
      acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], 1);
    }
    if (sub == 0 && t < ntl) {
#pragma unroll
      for (int g = 0; g < G; ++g) sS[g * a.tpc + t] = sValid[t] ? acc[g] * L.scale : kNegInf;
      const int li = sLog[t];
      if (pl.active && li >= 0) {
        if (li < S) leaderE[(size_t)h * a.s_cap + li] = acc[G];
        else set_status(st, HC_DEV_INDEX);
      }
    }
  }
  cluster.sync();

  // ---- leader: policy score, selection, compaction plan ------------------------------------
  if (rank == 0 && pl.active) {
    const bool snap = L.policy == HC_POLICY_SNAPKV;
    if (snap) {
      for (int hh = warp; hh < L.Hk; hh += kStepThreads / 32) {
        float* lg = sE + (size_t)hh * a.s_cap;
        float m = kNegInf;
        for (int t = lane; t < S; t += 32) {
          lg[t] = lg[t] * L.scale;  // the single observation row sees every key
          m = fmaxf(m, lg[t]);
        }
        m = warp_max(m);
        float l = 0.f;
        for (int t = lane; t < S; t += 32) l += __expf(lg[t] - m);
        l = warp_sum(l);
        for (int t = lane; t < S; t += 32) sImp[(size_t)hh * a.s_cap + t] = __expf(lg[t] - m) / l;
      }
      __syncthreads();
      const int pad = L.pool_kernel > 1 ? L.pool_kernel / 2 : 0;
      for (int t = tid; t < S; t += kStepThreads) {
        float tot = 0.f;
        for (int hh = 0; hh < L.Hk; ++hh) {
          const float* imp = sImp + (size_t)hh * a.s_cap;
          float v;
          if (pad == 0) {
            v = imp[t];
          } else if (L.pooling == HC_POOL_MAX) {
            v = kNegInf;
            for (int u = max(0, t - pad); u <= min(S - 1, t + pad); ++u) v = fmaxf(v, imp[u]);
          } else {
            v = 0.f;
            for (int u = max(0, t - pad); u <= min(S - 1, t + pad); ++u) v += imp[u];
            v /= (float)L.pool_kernel;
          }
          tot += v;
        }
        sTok[t] = tot / (float)L.Hk;
      }
    } else {
      const float inv = 1.f / sqrtf((float)L.D);
      for (int t = tid; t < S; t += kStepThreads) {
        float acc = 0.f;
        for (int hh = 0; hh < L.Hk; ++hh) acc += sE[(size_t)hh * a.s_cap + t] * inv;
        sTok[t] = acc / (float)L.Hk;
      }
    }
    __syncthreads();
    block_topk_flags([&](int i) { return sTok[i]; }, pl.prefix, pl.ntop, sSel, sTopk);
    for (int i = tid; i < (a.s_cap + 31) / 32; i += kStepThreads) sEvMask[i] = 0u;
    __syncthreads();
    const int n_ev_total = pl.prefix - pl.ntop;
    const int cold_head = st->cold_head, cold_count = st->cold_count;
    int kept = 0, evicted = 0;
    for (int base = 0; base < S; base += kStepThreads) {
      const int t = base + tid;
      int keep = 0, ev = 0, phys = -1;
      if (t < S) {
        keep = (t >= pl.prefix) || sSel[t];
        ev = !keep;
        phys = t < n_hot ? sOldOrd[t] : new_slot;
      }
      int tk2, te2;
      const int rk = block_exclusive_scan(keep, sTopk + 256, tk2);
      const int re = block_exclusive_scan(ev, sTopk + 256, te2);
      if (t < S) {
        if (keep) {
          sOrd[kept + rk] = phys;
        } else {
          const int j = evicted + re;
          sEvList[2 * j] = phys;
          sEvList[2 * j + 1] = (j >= n_ev_total - d.ccap) ? (int)(((long)cold_head + cold_count + j) % d.ccap) : -1;
          atomicOr(&sEvMask[t >> 5], 1u << (t & 31));
        }
      }
      kept += tk2;
      evicted += te2;
    }
    if (tid == 0) sMisc[0] = evicted;
    __syncthreads();
    // new logical order and freed slots (the new token's slot left the stack: n_free - 1)
    for (int i = tid; i < kept; i += kStepThreads) d.hot_ord[i] = sOrd[i];
    for (int j = tid; j < evicted; j += kStepThreads)
      if (n_free - 1 + j < d.cap) d.hot_free[n_free - 1 + j] = sEvList[2 * j];
  } else if (rank == 0 && tid == 0) {
    sMisc[0] = 0;
  }
  cluster.sync();

  // ---- attention partial without the evicted tokens ------------------------------------------
  const uint32_t* remMask = cluster.map_shared_rank(sEvMask, 0);
  const int n_ev = *cluster.map_shared_rank(sMisc, 0);
  if (pl.active && n_ev > 0) {
    for (int t = tid; t < ntl; t += kStepThreads) {
      const int li = sLog[t];
      if (li >= 0 && ((remMask[li >> 5] >> (li & 31)) & 1u)) {
        for (int g = 0; g < G; ++g) sS[g * a.tpc + t] = kNegInf;
      }
    }
    // this CTA's share of the evicted payloads (copied after the last cluster barrier, so the
    // leader never waits for them): token j goes to rank ncta-1-(j mod ncta)
    const int* remList = cluster.map_shared_rank(sEvList, 0);
    const int mine0 = ncta - 1 - rank;
    const int qmax = a.s_cap / kStepMaxCluster + 2;
    for (int q = tid; mine0 + q * ncta < n_ev && q < qmax; q += kStepThreads) {
      const int j = mine0 + q * ncta;
      sEvCopy[2 * q] = remList[2 * j];
      sEvCopy[2 * q + 1] = remList[2 * j + 1];
    }
  }
  __syncthreads();
  for (int g = warp; g < G; g += kStepThreads / 32) {
    float m = kNegInf;
    for (int t = lane; t < ntl; t += 32) m = fmaxf(m, sS[g * a.tpc + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < ntl; t += 32) {
      const float x = sS[g * a.tpc + t];
      const float pr = (x == kNegInf) ? 0.f : __expf(x - m);
      sS[g * a.tpc + t] = pr;
      l += pr;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sML[g] = m;
      sML[G + g] = l;
    }
  }
  if (!__syncthreads_and(mbar_wait(&bars[1], 0))) {
    if (tid == 0) set_status(st, HC_DEV_TIMEOUT);
  }
  // P.V: threads (d, half): half 0 takes even rows, half 1 odd rows, then add
  constexpr int PSTRIDE = G * D + 2 * G;
  float* headLeaderPart = cluster.map_shared_rank(sPart, h * a.P) + (size_t)p * PSTRIDE;
  {
    const int dd = tid % D, half = tid / D;  // kStepThreads == 2*D for D=128; D=64 uses 4 quarters
    const int nsplit = kStepThreads / D;
    float o[G];
#pragma unroll
    for (int g = 0; g < G; ++g) o[g] = 0.f;
    for (int t = half; t < ntl; t += nsplit) {
      const float vv = E::to_f(sV[(size_t)t * D + dd]);
#pragma unroll
      for (int g = 0; g < G; ++g) o[g] = fmaf(sS[g * a.tpc + t], vv, o[g]);
    }
    __syncthreads();
    // fold the splits through this CTA's sS area (scores are no longer needed)
    float* red = sS;
    if (half > 0)
#pragma unroll
      for (int g = 0; g < G; ++g) red[((size_t)(half - 1) * G + g) * D + dd] = o[g];
    __syncthreads();
    if (half == 0) {
      for (int k2 = 1; k2 < nsplit; ++k2)
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] += red[((size_t)(k2 - 1) * G + g) * D + dd];
#pragma unroll
      for (int g = 0; g < G; ++g) headLeaderPart[g * D + dd] = o[g];
    }
    if (tid < 2 * G) headLeaderPart[G * D + tid] = sML[tid];
  }
  cluster.sync();

  // ---- head leaders merge the P partials ------------------------------------------------------
  if (p == 0) {
    T* outp = reinterpret_cast<T*>(a.out) + ((size_t)s * L.Hq + (size_t)h * G) * D;
    for (int i = tid; i < G * D; i += kStepThreads) {
      const int g = i / D, dd = i % D;
      float Mx = kNegInf;
      for (int q = 0; q < a.P; ++q) Mx = fmaxf(Mx, sPart[(size_t)q * PSTRIDE + G * D + g]);
      float Ls = 0.f, Os = 0.f;
      for (int q = 0; q < a.P; ++q) {
        const float* pc = sPart + (size_t)q * PSTRIDE;
        const float w = __expf(pc[G * D + g] - Mx);
        Ls = fmaf(pc[G * D + G + g], w, Ls);
        Os = fmaf(pc[g * D + dd], w, Os);
      }
      float r = Os / Ls;
      if (a.overflow_nan && Mx >= kExpOverflow) r = __int_as_float(0x7fc00000);
      outp[(size_t)g * D + dd] = E::from_f(r);
    }
  }
  // ---- counters (one thread of the leader) -------------------------------------------------------
  if (rank == 0 && tid == 0) {
    // the new token: position of its slot, and its logical entry when nothing was compressed
    // (a compression rewrote the whole order above)
    d.hot_pos[new_slot] = cur_pos;
    if (!pl.active) d.hot_ord[n_hot] = new_slot;
    const int ev = pl.active ? sMisc[0] : 0;
    if (ev > 0) {
      const long total = (long)st->cold_count + ev;
      if (total > d.ccap) {
        st->cold_head = (int)(((long)st->cold_head + total - d.ccap) % d.ccap);
        st->cold_count = d.ccap;
      } else {
        st->cold_count = (int)total;
      }
    }
    st->n_evict = ev;
    st->n_hot = S - ev;
    st->n_free = n_free - 1 + ev;
    if (d.p_max > 0) st->qwin_head = (qwin_slot + 1) % d.p_max;
  }
  // ---- work nothing in this kernel waits for ---------------------------------------------------
  if (pl.active && n_ev > 0) {
    const int mine0 = ncta - 1 - rank;
    const int nmine = mine0 < n_ev ? min(a.s_cap / kStepMaxCluster + 2, (n_ev - mine0 + ncta - 1) / ncta) : 0;
    for (int q = warp; q < nmine; q += kStepThreads / 32) step_evict_one<DT, D>(L, d, sEvCopy[2 * q], sEvCopy[2 * q + 1]);
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
  pdl_launch_dependents();
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
int step_parts(int Hk) { return (Hk >= 1 && Hk <= kStepMaxCluster && kStepMaxCluster % Hk == 0) ? kStepMaxCluster / Hk : 0; }

size_t step_smem_bytes(const hc_layer& L, int use_held) {
  const int P = step_parts(L.Hk);
  if (!P) return 0;
  const int esz = L.dtype == HC_F32 ? 4 : 2;
  const int G = L.Hq / L.Hk;
  const int tokens = (use_held ? L.max_r : 0) + L.max_cap;
  const int tpc = (tokens + P - 1) / P;
  return step_smem(L.D, esz, G, tpc, L.max_cap, P, L.Hk).total;
}

template <int DT, int D, int G>
static cudaError_t step_t(const StepArgs& a, cudaStream_t stream) {
  using T = typename Elem<DT>::T;
  const StepSmem M = step_smem(D, sizeof(T), G, a.tpc, a.s_cap, a.P, a.L.Hk);
  auto kern = step_kernel<DT, D, G>;
  cudaError_t e = ensure_smem(kern, M.total);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.L.Hk * a.P, a.L.n_seq);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = M.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.L.Hk * a.P;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
  if (e != cudaSuccess) return e;
  if (clusters < 1) return cudaErrorNotSupported;
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
  return cudaErrorInvalidValue;
}

cudaError_t launch_step(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                        const void* c, const void* sn, const int64_t* pos, int use_held, void* out, int overflow_nan,
                        cudaStream_t stream) {
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
  a.P = step_parts(L.Hk);
  if (!a.P) return cudaErrorNotSupported;
  const int tokens = (use_held ? L.max_r : 0) + L.max_cap;
  a.tpc = (tokens + a.P - 1) / a.P;
  a.s_cap = L.max_cap;
  if (L.dtype == HC_F32 && L.D == 128) return step_g<HC_F32, 128>(a, stream);
  if (L.dtype == HC_F16 && L.D == 128) return step_g<HC_F16, 128>(a, stream);
  if (L.dtype == HC_BF16 && L.D == 128) return step_g<HC_BF16, 128>(a, stream);
  if (L.dtype == HC_F32 && L.D == 64) return step_g<HC_F32, 64>(a, stream);
  if (L.dtype == HC_F16 && L.D == 64) return step_g<HC_F16, 64>(a, stream);
  if (L.dtype == HC_BF16 && L.D == 64) return step_g<HC_BF16, 64>(a, stream);
  return cudaErrorInvalidValue;
}

}  // namespace hc
