// Fused decode step of one layer: append, compression with eviction into the cold ring, and
// attention over [held | hot] in one launch — one thread-block cluster of 16 CTAs per sequence.
//
// The reference runs this as a chain of torch ops and a Triton kernel per layer
// (patch.py:161-305 with cache.py:130-151 and cache.py:37-128). Split into separate kernels
// (hc_append, hc_compress, hc_attend) the step pays a launch and a global round trip per
// stage; at batch 1 that latency, not HBM bandwidth, sets the time. Here CTA (h, p) of the
// cluster owns KV head h and part p of P = 16/Hk parts of head h's rows in PHYSICAL order,
// [held rows 0..r_max) ++ [slab slots 0..cap): order does not matter to attention, and
// physical order makes each part contiguous in HBM.
//   1. Warp 0 starts TMA copies of the part's K rows (tensor boxes into the swizzled MMA layout)
//      and V rows (bulk copies) — before the dependency wait when the launch before this one
//      left the layer's state alone — while the CTA reads the counters and order table, maps
//      its slots to logical indices (free slots stay unmapped and are masked), and RoPEs the new
//      token's query heads of its group and, if the new slot is its own, the new key.
//   2. Scoring with tcgen05 (16-bit types; CUDA cores for f32): G attention logits and the
//      eviction logit (GQA-mean query . k) per row. Eviction logits go, by logical index, to
//      every CTA of the cluster, with every warp's softmax statistics of them (barrier A).
//   3. While barrier A completes, every warp computes its flash-decode partial (max, sum, P.V)
//      over its 32 rows.
//   4. Policy: every CTA combines each head's statistics, scores every prefix token (SnapKV
//      softmax and pooling, or the raw hot/cold logit; mean over heads) and takes the lowest
//      (ties: the higher index) — the same arithmetic on the same data, so every CTA selects
//      the same token with no further exchange. The warp holding the evicted row subtracts it
//      from its partial (or recomputes without it where the row carried most of the mass).
//      More than one eviction ranks every prefix token against all keys (one more exchange)
//      and the warps recompute their partials.
//   5. The warps' partials are combined per column and each column block goes to the CTA of
//      head h that finalizes it (last barrier). Owners of 32-token words compact the logical
//      order and push freed slots; evicted payloads are copied into the cold ring with their
//      index vectors; the last CTA pushes the query pool.
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
  int P;      // parts per KV head; cluster = Hk * P = 16
  int chunk;  // physical rows per CTA (multiple of 8)
  int krows;  // rows of the K area: with tensor-core scoring, whole 128-row tiles and the slack of
              // the last 64-row TMA box
  int r8;     // held rows in the physical order, a multiple of 8 (rows past r_max are masked)
  int vrows;  // rows of the V area: with tensor-core P.V, the 16-row boxes' slack included
  int xs;     // floats per CTA in the exchange: its rows' eviction logits, then 16 warps' statistics
  int s_cap;  // hot tokens at most
  int wpc;    // 32-token words a CTA owns at most
};

__host__ __device__ inline StepGeom step_geom(int Hk, int max_cap, int max_r, int use_held, bool mma, bool pv_mma) {
  StepGeom g{};
  g.P = (Hk >= 1 && Hk <= kStepMaxCluster && kStepMaxCluster % Hk == 0) ? kStepMaxCluster / Hk : 0;
  if (!g.P) return g;
  g.s_cap = max_cap;
  g.r8 = use_held ? (max_r + 7) & ~7 : 0;
  const int rows = g.r8 + max_cap;
  g.chunk = (((rows + g.P - 1) / g.P) + 7) & ~7;
  g.krows = mma ? ((g.chunk + 64 + 127) & ~127) : g.chunk;
  g.vrows = pv_mma ? g.chunk + 16 : g.chunk;
  g.xs = g.chunk + 2 * kStepWarps;
  g.wpc = ((max_cap + 31) / 32 + kStepMaxCluster - 1) / kStepMaxCluster;
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
  int early;  // HC_STEP_EARLY_* bits: state this launch may read before its dependency wait
  StepGeom g;
};

struct StepSmem {
  size_t k, qb, v, q, knew, vn, a, inv, ord, fre, held, xch, loc, wst, key, red, mask, evl, o, ml, misc, tmem, bars,
      total;
};

__host__ __device__ inline size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

__host__ __device__ inline size_t step_words(int s_cap) { return (size_t)(s_cap + 31) / 32; }

__host__ __device__ inline StepSmem step_smem(int D, int esz, int G, int Hk, int max_r, const StepGeom& g) {
  StepSmem m{};
  size_t o = 0;
  auto take = [&](size_t b) { size_t r = o; o += al16(b); return r; };
  // K rows of this CTA's part (16-bit: D/64 planes of 128-byte swizzled rows, 1024-aligned);
  // after scoring the same area holds the warps' P.V partials, probabilities and statistics
  const size_t kb = (size_t)g.krows * D * esz;
  const size_t rb = (size_t)kStepWarps * G * (D + 32 + 2) * 4;
  m.k = take(kb > rb ? kb : rb);
  o = (o + 1023) & ~size_t(1023);
  m.qb = take((size_t)16 * D * esz);  // MMA query operand: G heads, the mean, zero rows (N = 16)
  // V rows: 16-bit, D/64 planes of 128-byte swizzled rows (1024-aligned) read by the P.V MMAs;
  // f32, plain rows
  m.v = take((size_t)g.vrows * D * esz);
  o = (o + 1023) & ~size_t(1023);
  m.q = take((size_t)(G + 1) * D * 4);       // RoPE'd query heads and their GQA mean
  m.knew = take((size_t)D * esz);            // the new key after RoPE
  m.vn = take((size_t)D * esz);              // the new value
  m.a = take((size_t)G * g.chunk * 4);       // attention logits, then probabilities
  m.inv = take((size_t)g.chunk * 4);         // logical index of each row, -1 when not attended
  m.ord = take((size_t)g.s_cap * 4);         // logical order (physical slot per logical index)
  m.fre = take((size_t)g.s_cap * 4);         // free-slot stack
  m.held = take((size_t)(max_r > 0 ? max_r : 1) * 4);  // held rows attended this step
  // exchange: every CTA's eviction logits by physical row and its warps' softmax statistics
  m.xch = take((size_t)kStepMaxCluster * g.xs * 4);
  m.loc = take((size_t)g.s_cap * 4);  // where each hot token's row sits in a head's exchange
  m.wst = take((size_t)2 * kStepWarps * G * 4);  // each warp's attention-logit maxima and sums
  m.key = take((size_t)g.s_cap * 4);         // policy score keys of the prefix, by logical index
  m.red = take((size_t)(4 * kStepMaxCluster + 4 * kStepWarps) * 8);
  m.mask = take(step_words(g.s_cap) * 4);    // evicted tokens, one bit per logical index
  m.evl = take((size_t)3 * g.wpc * 32 * 4);  // evicted tokens of the words this CTA owns
  m.o = take((size_t)G * D * 4);             // partials of this CTA's column block from every part
  m.ml = take((size_t)2 * G * kStepMaxCluster * 4);
  m.misc = take(64);
  m.tmem = take(16);
  m.bars = take(48);
  m.total = o + 1024;  // room to align the dynamic shared memory base to 1024 bytes
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

// Index vector and position of one evicted token (controller.py:178-182, 200-212): mean over
// heads of the pre-RoPE key, L2-normalised, zero-padded to F; one warp.
template <int DT, int D>
__device__ void step_evict_vec(const hc_layer& L, const hc_seq_desc& d, int slot, int dst, int64_t posv) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int PER = (D + 31) / 32;
  const int lane = threadIdx.x & 31;
  float mean[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) mean[i] = 0.f;
  for (int h0 = 0; h0 < L.Hk; h0 += 8) {
    const int nh = min(8, L.Hk - h0);
    T kr[8][PER];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nh) break;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int dd = lane + 32 * i;
        if (dd < D) kr[j][i] = reinterpret_cast<const T*>(d.hot_kpre)[((size_t)(h0 + j) * d.cap + slot) * D + dd];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nh) break;
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (lane + 32 * i < D) mean[i] += E::to_f(kr[j][i]);
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
  constexpr int ROWB = D * ESZ;
  constexpr int KCH = ROWB / 16;  // 16-byte chunks per row
  constexpr int VE = 16 / ESZ;    // elements per chunk
  constexpr int CPL = KCH / 8;    // chunks per lane when 8 lanes share a row
  constexpr int EPL = CPL * VE;   // elements per lane
  constexpr int H = D / 2;
  constexpr int RP = ((G + 1) * H + kStepThreads - 1) / kStepThreads;  // RoPE pairs per thread
  constexpr bool QREG = (G + 1) * EPL <= 80;  // query rows kept in registers while scoring (fp32)
  constexpr bool MMA = DT != HC_F32;          // 16-bit: tcgen05 scoring on TMA-loaded, swizzled K
  constexpr int N8 = 16;                      // MMA N (M = 128 takes N in steps of 16): heads + mean, padded
  constexpr int NL = ((G + 1 + 7) / 8) * 8;   // accumulator columns read back
  constexpr int PL = D / 64;                  // 128-byte planes of a K row
  // P.V on the tensor cores (16-bit, D = 128: M = D = 128 lanes of O^T, N = 16 query columns):
  // V arrives in the swizzled planes the MMA reads as its MN-major A operand
  constexpr bool PVMMA = MMA && D == 128;
  constexpr uint32_t kFmt = DT == HC_BF16 ? 1u : 0u;
  // instruction descriptor: f32 accumulate, A and B of the layer's type, N = 16, M = 128, K-major
  constexpr uint32_t kIdesc = (1u << 4) | (kFmt << 7) | (kFmt << 10) | ((uint32_t)(N8 >> 3) << 17) |
                              ((uint32_t)(128 >> 4) << 24);
  static_assert(KCH % 8 == 0, "rows must be a multiple of 128 bytes");
  static_assert(G + 1 <= 16, "query heads per KV head");
  cg::cluster_group cluster = cg::this_cluster();
  const hc_layer& L = a.L;
  const StepGeom& gm = a.g;
  const int rank = (int)cluster.block_rank();
  const int P = gm.P, ncta = L.Hk * P;
  const int h = rank / P, p = rank % P;
  const int s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int chunk = gm.chunk;

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const StepSmem M = step_smem(D, ESZ, G, L.Hk, L.max_r, gm);
  T* sK = reinterpret_cast<T*>(smem + M.k);
  T* sQb = reinterpret_cast<T*>(smem + M.qb);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + M.tmem);
  T* sV = reinterpret_cast<T*>(smem + M.v);
  float* sQ = reinterpret_cast<float*>(smem + M.q);
  T* sKnew = reinterpret_cast<T*>(smem + M.knew);
  T* sVn = reinterpret_cast<T*>(smem + M.vn);
  float* sA = reinterpret_cast<float*>(smem + M.a);
  int* sInv = reinterpret_cast<int*>(smem + M.inv);
  int* sOrd = reinterpret_cast<int*>(smem + M.ord);
  int* sFree = reinterpret_cast<int*>(smem + M.fre);
  int* sHeld = reinterpret_cast<int*>(smem + M.held);
  float* sX = reinterpret_cast<float*>(smem + M.xch);  // [cluster rank][xs]
  int* sLoc = reinterpret_cast<int*>(smem + M.loc);     // [logical index]: part * xs + row
  float* sWst = reinterpret_cast<float*>(smem + M.wst);    // [warp][G] maxima, then [warp][G] sums
  uint32_t* sKey = reinterpret_cast<uint32_t*>(smem + M.key);
  float* sRed = reinterpret_cast<float*>(smem + M.red);  // per-warp partials and per-head statistics
  uint32_t* sMask = reinterpret_cast<uint32_t*>(smem + M.mask);
  int* sEvl = reinterpret_cast<int*>(smem + M.evl);
  float* sO = reinterpret_cast<float*>(smem + M.o);
  float* sML = reinterpret_cast<float*>(smem + M.ml);
  int* sMisc = reinterpret_cast<int*>(smem + M.misc);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + M.bars);

  // the descriptor is written once when the layer is set up, so it is read before the wait
  const hc_seq_desc d = L.desc[s];
  // this part's rows: physical index u in [held rows 0..R) ++ [slots 0..cap)
  const int R = a.use_held ? gm.r8 : 0;  // held rows, padded to 8; rows past r_max are masked
  const int Un = R + d.cap;
  const int u0 = min(p * chunk, Un), u1 = min(u0 + chunk, Un), nrows = u1 - u0;
  const int hb = u0, nh = max(0, min(u1, R) - hb);          // held rows [hb, hb + nh), nh % 8 == 0
  const int nhr = max(0, min(hb + nh, d.r_max) - hb);       // of which real held rows
  const int sb = max(u0, R) - R, ns = max(0, u1 - max(u0, R));  // slots [sb, sb + ns)
  const int cap = d.cap;
  // What may be read before the dependency wait: the host sets these bits when the launch
  // preceding this one on the stream wrote none of that state of this layer (the layer's own
  // previous step finished before that launch started). The new token's inputs are always
  // read after the wait: the preceding kernel of a model produces them.
  const bool early_hot = (a.early & HC_STEP_EARLY_HOT) != 0;    // slab K/V, order table, free stack
  const bool early_held = (a.early & HC_STEP_EARLY_HELD) != 0;  // held K/V rows and their flags

  // ---- copies of this part's K and V rows, issued by warp 0: for 16-bit types TMA tensor boxes
  //      into the swizzled layout the MMAs read (K: 64-row slot boxes; V: 16-row slot boxes, so
  //      that the V area needs little slack; 8-row boxes for held rows), for f32 bulk copies ----
  const int nhb = nh >> 3, nsb = (ns + 63) >> 6, nsv = (ns + 15) >> 4;
  if (warp == 0) {
    if (lane == 0) {
      mbar_init(&bars[0], 1);
      mbar_init(&bars[1], 1);
      mbar_init(&bars[2], 1);
      mbar_init(&bars[3], 1);
      mbar_init(&bars[4], 1);  // the exchange: peers' copies complete on it
      fence_mbar_init();
      const uint32_t vbytes = (uint32_t)((nhr + ns) * ROWB);
      mbar_arrive_expect_tx(&bars[0], MMA ? (uint32_t)((nh + 64 * nsb) * 128 * PL) : vbytes);
      mbar_arrive_expect_tx(&bars[1], PVMMA ? (uint32_t)((nh + 16 * nsv) * 128 * PL) : vbytes);
    }
    __syncwarp();
  }
  // arrival: this CTA has started and initialised its barriers; waited on before the first
  // distributed shared memory access
  cluster_arrive_relaxed();
  auto issue_rows = [&](bool held) {
    // warp 0 only: the K boxes of the held rows or of the slab slots, then their V copy
    if constexpr (MMA) {
      const char* kmaps = reinterpret_cast<const char*>(L.kmaps);
      const int y_held = (s * L.Hk + h) * d.r_max + hb;
      const int y_hot = (s * L.Hk) * L.max_cap + h * d.cap + sb;
      const int nb = held ? nhb : nsb;
      for (int b = lane; b < nb * PL; b += 32) {
        const int pl = b / nb, j = b - pl * nb;
        unsigned char* plane = reinterpret_cast<unsigned char*>(sK) + (size_t)pl * gm.krows * 128;
        if (held) tma_load_2d(plane + (size_t)j * 8 * 128, kmaps + 128, pl * 64, y_held + 8 * j, &bars[0]);
        else tma_load_2d(plane + (size_t)(nh + 64 * j) * 128, kmaps, pl * 64, y_hot + 64 * j, &bars[0]);
      }
      if constexpr (PVMMA) {
        const int nbv = held ? nhb : nsv;
        for (int b = lane; b < nbv * PL; b += 32) {
          const int pl = b / nbv, j = b - pl * nbv;
          unsigned char* plane = reinterpret_cast<unsigned char*>(sV) + (size_t)pl * gm.vrows * 128;
          if (held) tma_load_2d(plane + (size_t)j * 8 * 128, kmaps + 384, pl * 64, y_held + 8 * j, &bars[1]);
          else tma_load_2d(plane + (size_t)(nh + 16 * j) * 128, kmaps + 256, pl * 64, y_hot + 16 * j, &bars[1]);
        }
      }
    } else {
      if (lane == 1 && held && nhr > 0)
        bulk_g2s(sK, reinterpret_cast<const T*>(d.held_k) + ((size_t)h * d.r_max + hb) * D, (uint32_t)(nhr * ROWB),
                 &bars[0]);
      if (lane == 2 && !held && ns > 0)
        bulk_g2s(sK + (size_t)nh * D, reinterpret_cast<const T*>(d.hot_k) + ((size_t)h * d.cap + sb) * D,
                 (uint32_t)(ns * ROWB), &bars[0]);
    }
    if constexpr (!PVMMA) {
      if (lane == 3 && held && nhr > 0)
        bulk_g2s(sV, reinterpret_cast<const T*>(d.held_v) + ((size_t)h * d.r_max + hb) * D, (uint32_t)(nhr * ROWB),
                 &bars[1]);
      if (lane == 4 && !held && ns > 0)
        bulk_g2s(sV + (size_t)nh * D, reinterpret_cast<const T*>(d.hot_v) + ((size_t)h * d.cap + sb) * D,
                 (uint32_t)(ns * ROWB), &bars[1]);
    }
  };
  if (warp == 0) {
    // the four maps: hot K slab, held K rows, hot V slab, held V rows
    if (MMA && lane >= 28) prefetch_tensormap(reinterpret_cast<const char*>(L.kmaps) + 128 * (lane - 28));
    if (early_held) issue_rows(true);
    if (early_hot) issue_rows(false);
  }
  // order table and free stack: all loads first, stores to shared memory later (one round trip)
  constexpr int kPre = 4;
  int ov[kPre], fv[kPre];
  auto load_order = [&]() {
#pragma unroll
    for (int j = 0; j < kPre; ++j) {
      const int i = tid + j * kStepThreads;
      if (i < cap) {
        ov[j] = d.hot_ord[i];
        fv[j] = d.hot_free[i];
      }
    }
  };
  const bool hv_ok = a.use_held && tid < d.r_max;
  uint8_t hval = 0;
  int64_t hpos = 0;
  auto row_of_slot = [&](int slot) { return (slot >= sb && slot < sb + ns) ? nh + slot - sb : -1; };
  // the exchange entry of a slot within a head's P parts: part * xs + row in the part
  auto loc_of_slot = [&](int slot) {
    const int u = R + slot, q = u / chunk;
    return q * gm.xs + (u - q * chunk);
  };
  // the hot tier's counters, order table and free stack into registers and shared memory, and the
  // logical index of every own slot row (free slots stay -1 and are masked)
  hc_seq_state* st = d.st;
  int n_hot = 0, n_free = 0, qwin_head = 0, cold_head = 0, cold_count = 0, held_len = 0;
  auto stage_hot = [&]() {
    n_hot = st->n_hot;
    n_free = st->n_free;
    qwin_head = st->qwin_head;
    cold_head = st->cold_head;
    cold_count = st->cold_count;
    load_order();
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
    for (int i = tid; i < chunk; i += kStepThreads) sInv[i] = -1;
    __syncthreads();
    for (int li = tid; li < min(n_hot, cap); li += kStepThreads) {
      const int slot = sOrd[li];
      if (slot < 0 || slot >= cap) {
        set_status(st, HC_DEV_INDEX);
        sLoc[li] = 0;
        continue;
      }
      const int i = row_of_slot(slot);
      if (i >= 0) sInv[i] = li;
      sLoc[li] = loc_of_slot(slot);
    }
  };
  if (early_hot) stage_hot();
  if (early_held) {
    held_len = st->held_len;
    if (hv_ok) {
      hval = d.held_valid[tid];
      hpos = d.held_pos[tid];
    }
  }
  // L2 prefetch of the state that is read after the wait (the launch before this one may still
  // write it: a prefetch only warms L2, which is safe for such lines)
  if (tid < 64) {
    const int nl_ord = (d.cap * 4 + 127) / 128, nl_pos = (d.r_max * 8 + 127) / 128;
    if (tid == 0) {
      if (!early_held && nhr > 0) {
        const size_t off = ((size_t)h * d.r_max + hb) * ROWB;
        bulk_prefetch_l2(reinterpret_cast<const char*>(d.held_k) + off, (uint32_t)(nhr * ROWB));
        bulk_prefetch_l2(reinterpret_cast<const char*>(d.held_v) + off, (uint32_t)(nhr * ROWB));
      }
      if (!early_hot && ns > 0) {
        const size_t off = ((size_t)h * d.cap + sb) * ROWB;
        bulk_prefetch_l2(reinterpret_cast<const char*>(d.hot_k) + off, (uint32_t)(ns * ROWB));
        bulk_prefetch_l2(reinterpret_cast<const char*>(d.hot_v) + off, (uint32_t)(ns * ROWB));
      }
      if (!early_held && a.use_held && d.held_valid) prefetch_l2(d.held_valid);
    } else if (!early_hot && tid <= nl_ord) {
      prefetch_l2(reinterpret_cast<const char*>(d.hot_ord) + (size_t)(tid - 1) * 128);
      prefetch_l2(reinterpret_cast<const char*>(d.hot_free) + (size_t)(tid - 1) * 128);
    } else if (!early_held && a.use_held && d.held_pos && tid > nl_ord && tid <= nl_ord + nl_pos) {
      prefetch_l2(reinterpret_cast<const char*>(d.held_pos) + (size_t)(tid - 1 - nl_ord) * 128);
    }
  }
  // L2 prefetch of the counters and of this step's inputs (the query rows of this head group, or
  // all of them for the CTA that pushes the query pool; the new key, value, cos/sin, position):
  // written by the preceding kernel in a model, so only warmed here and read after the wait. A
  // prefetch only warms L2, so it is safe for lines that kernel still writes.
  if (tid >= 64) {
    const int lt = tid - 64;
    const int rb = D * ESZ;  // bytes of one head row
    const bool all_q = rank == ncta - 1;
    const int nq = ((all_q ? L.Hq : G) * rb + 127) / 128, nr = (rb + 127) / 128;
    const char* qrow = reinterpret_cast<const char*>(a.q_pre) + (size_t)s * a.qss * ESZ + (all_q ? 0 : (size_t)h * G * rb);
    if (lt < nq) {
      prefetch_l2(qrow + (size_t)lt * 128);
    } else if (lt < nq + nr) {
      prefetch_l2(reinterpret_cast<const char*>(a.k_pre) + ((size_t)s * a.kvss + (size_t)h * D) * ESZ +
                  (size_t)(lt - nq) * 128);
    } else if (lt < nq + 2 * nr) {
      prefetch_l2(reinterpret_cast<const char*>(a.v) + ((size_t)s * a.kvss + (size_t)h * D) * ESZ +
                  (size_t)(lt - nq - nr) * 128);
    } else if (a.cos && lt < nq + 3 * nr) {
      prefetch_l2(reinterpret_cast<const char*>(a.cos) + (size_t)s * rb + (size_t)(lt - nq - 2 * nr) * 128);
    } else if (a.sin && lt < nq + 4 * nr) {
      prefetch_l2(reinterpret_cast<const char*>(a.sin) + (size_t)s * rb + (size_t)(lt - nq - 3 * nr) * 128);
    } else if (lt == nq + 4 * nr) {
      prefetch_l2(a.pos + s);
    } else if (lt == nq + 4 * nr + 1) {
      prefetch_l2(d.st);
    }
  }
  pdl_wait();

  if (warp == 0) {
    if (!early_held) issue_rows(true);
    if (!early_hot) issue_rows(false);
  }
  if (!early_held) {
    held_len = st->held_len;
    if (hv_ok) {
      hval = d.held_valid[tid];
      hpos = d.held_pos[tid];
    }
  }
  // ---- the new token's inputs (with the hot tier's state, when it is read after the wait, in
  //      the same round trip) ----
  const int64_t cur_pos = a.pos[s];
  const T* __restrict__ qp = reinterpret_cast<const T*>(a.q_pre) + (size_t)s * a.qss;
  const T* __restrict__ kp = reinterpret_cast<const T*>(a.k_pre) + (size_t)s * a.kvss + (size_t)h * D;
  const T* __restrict__ vp = reinterpret_cast<const T*>(a.v) + (size_t)s * a.kvss + (size_t)h * D;
  // raw loads first (all in flight together), conversions after
  T xr[RP][2], cr[RP][2], sr[RP][2];
  float rx[RP][2], rc[RP][2], rs[RP][2];
  const bool have_cs = a.cos != nullptr;
#pragma unroll
  for (int j = 0; j < RP; ++j) {
    const int k = tid + j * kStepThreads;
    if (k < (G + 1) * H) {
      const int g = k / H, i = k % H;
      const T* x = g < G ? qp + (size_t)(h * G + g) * D : kp;
      xr[j][0] = x[i];
      xr[j][1] = x[i + H];
      if (have_cs) {
        const T* cs = reinterpret_cast<const T*>(a.cos) + (size_t)s * D;
        const T* sn = reinterpret_cast<const T*>(a.sin) + (size_t)s * D;
        cr[j][0] = cs[i];
        cr[j][1] = cs[i + H];
        sr[j][0] = sn[i];
        sr[j][1] = sn[i + H];
      } else {
        rc[j][0] = L.inv_freq[i];
      }
    }
  }
  const T vnew = tid < D ? vp[tid] : E::from_f(0.f);
  if (!early_hot) stage_hot();
  // the last CTA stages the query rows for the query-pool push
  const bool qpush = rank == ncta - 1 && d.p_max > 0;
  float qsum = 0.f;  // this thread's column of the query pool's new entry (the last CTA)
  if (qpush && tid < D)
    for (int hh = 0; hh < L.Hq; ++hh) qsum += E::to_f(qp[(size_t)hh * D + tid]);
#pragma unroll
  for (int j = 0; j < RP; ++j) {
    if (tid + j * kStepThreads < (G + 1) * H) {
      rx[j][0] = E::to_f(xr[j][0]);
      rx[j][1] = E::to_f(xr[j][1]);
      if (have_cs) {
        rc[j][0] = E::to_f(cr[j][0]);
        rc[j][1] = E::to_f(cr[j][1]);
        rs[j][0] = E::to_f(sr[j][0]);
        rs[j][1] = E::to_f(sr[j][1]);
      }
    }
  }
  if (hv_ok) sHeld[tid] = hval != 0 && hpos <= cur_pos;
  if (a.use_held)
    for (int t = tid + kStepThreads; t < d.r_max; t += kStepThreads)
      sHeld[t] = d.held_valid[t] != 0 && d.held_pos[t] <= cur_pos;
  if (tid == 0) sMisc[4] = 0;
  __syncthreads();

  const int n_held = a.use_held ? max(0, min(held_len, d.r_max)) : 0;
  const int new_slot = (n_free > 0 && n_free <= cap) ? sFree[n_free - 1] : -1;

  const int S = n_hot + 1;  // hot tokens after the append (logical index n_hot is the new one)
  // every CTA reads the same counters (nothing writes them before the last barrier): a
  // uniform exit, after this CTA's copies have landed
  if (n_hot < 0 || S > cap || S > gm.s_cap || new_slot < 0 || new_slot >= cap) {
    if (rank == 0 && tid == 0) set_status(st, HC_DEV_CAPACITY);
    const bool k_ok = mbar_wait(&bars[0], 0);
    const bool v_ok = mbar_wait(&bars[1], 0);
    if (!(k_ok && v_ok) && tid == 0) set_status(st, HC_DEV_TIMEOUT);
    cluster_wait();
    return;
  }
  const Plan pl = step_plan(L, d.budget, S);
  const int n_ev_plan = pl.active ? pl.prefix - pl.ntop : 0;
  const bool policy = pl.active && n_ev_plan > 0;
  // the exchange brings one block from every other CTA of the cluster
  if (policy && tid == 0) mbar_arrive_expect_tx(&bars[4], (uint32_t)((ncta - 1) * gm.xs * 4));
  const int nwords = (S + 31) >> 5;
  // CTA r owns the 32-token words w with w * ncta / nwords == r: it writes their entries of the
  // order table and free stack and copies their evicted tokens into the cold ring
  const int w0 = (rank * nwords + ncta - 1) / ncta, w1 = ((rank + 1) * nwords + ncta - 1) / ncta;
  const int own0 = w0 * 32, own_n = max(0, min(w1 * 32, S) - own0), nw_own = w1 - w0;
  const int qwin_slot = d.p_max > 0 ? ((qwin_head % d.p_max) + d.p_max) % d.p_max : 0;
  // query pool push: mean over all query heads of the pre-RoPE query (controller.py:240-241)
  if (qpush && tid < D) reinterpret_cast<T*>(d.qwin)[(size_t)qwin_slot * D + tid] = E::from_f(qsum / (float)L.Hq);
  auto phys_of = [&](int li) { return li < n_hot ? sOrd[li] : new_slot; };
  const int i_new = row_of_slot(new_slot);
  if (tid == 0) {
    if (i_new >= 0) sInv[i_new] = n_hot;
    sLoc[n_hot] = loc_of_slot(new_slot);
  }

  // ---- RoPE of the new token (patch.py:161-162) while the copies are in flight --------------
#pragma unroll
  for (int j = 0; j < RP; ++j) {
    const int k = tid + j * kStepThreads;
    if (k >= (G + 1) * H) continue;
    const int g = k / H, i = k % H;
    if (g == G && i_new < 0) continue;
    float c0, s0, c1, s1;
    if (a.cos) {
      c0 = rc[j][0];
      c1 = rc[j][1];
      s0 = rs[j][0];
      s1 = rs[j][1];
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
    } else {
      const T k0 = E::from_f(o0), k1 = E::from_f(o1);
      sKnew[i] = k0;
      sKnew[i + H] = k1;
      // the owner of the new slot writes its slab rows for head h (cache.py:145-148)
      const size_t off = ((size_t)h * cap + new_slot) * D + i;
      reinterpret_cast<T*>(d.hot_k)[off] = k0;
      reinterpret_cast<T*>(d.hot_k)[off + H] = k1;
      reinterpret_cast<T*>(d.hot_kpre)[off] = E::from_f(rx[j][0]);
      reinterpret_cast<T*>(d.hot_kpre)[off + H] = E::from_f(rx[j][1]);
    }
  }
  if (i_new >= 0 && tid < D) {
    reinterpret_cast<T*>(d.hot_v)[((size_t)h * cap + new_slot) * D + tid] = vnew;
    sVn[tid] = vnew;
  }
  __syncthreads();
  // GQA-mean query of this KV head, rounded to the dtype (cache.py:60-64 / scoring.py:17-26)
  for (int dd = tid; dd < D; dd += kStepThreads) {
    float acc = 0.f;
#pragma unroll
    for (int g = 0; g < G; ++g) acc += sQ[g * D + dd];
    sQ[G * D + dd] = E::round(acc / (float)G);
  }
  // K rows landed: the new key replaces the stale copy of its slot
  if (!__syncthreads_and(mbar_wait(&bars[0], 0)) && tid == 0) set_status(st, HC_DEV_TIMEOUT);
  if (i_new >= 0)
    for (int i = tid; i < D; i += kStepThreads) {
      if constexpr (MMA) {
        // row i_new of plane i/64, 16-byte chunk swizzled by the row (the TMA's 128-byte pattern)
        const int c = (i & 63) >> 3;
        reinterpret_cast<T*>(reinterpret_cast<unsigned char*>(sK) + (size_t)(i >> 6) * gm.krows * 128 +
                             (size_t)i_new * 128 + ((c ^ (i_new & 7)) << 4))[i & 7] = sKnew[i];
      } else {
        sK[(size_t)i_new * D + i] = sKnew[i];
      }
    }
  if constexpr (MMA) {
    // B operand: N8 rows (query heads, their mean, zeros) x D, K-major, 128-byte swizzle
    for (int k = tid; k < N8 * D; k += kStepThreads) {
      const int n = k / D, i = k % D, c = (i & 63) >> 3;
      reinterpret_cast<T*>(reinterpret_cast<unsigned char*>(sQb) + (size_t)(i >> 6) * N8 * 128 + (size_t)n * 128 +
                           ((c ^ (n & 7)) << 4))[i & 7] = E::from_f(n <= G ? sQ[n * D + i] : 0.f);
    }
    fence_proxy_async_smem();  // generic writes above are read by the tensor cores
  }
  __syncthreads();

  // ---- scoring: G attention logits + the eviction logit (GQA-mean query . k) per row --------
  cluster_wait();  // every CTA of the cluster has started
  const bool snap = L.policy == HC_POLICY_SNAPKV;
  // running softmax statistics (max, sum rescaled to it) of the scaled eviction logits of the
  // rows this thread scores (SnapKV: the single observation row sees every key)
  float em = kNegInf, el = 0.f;
  auto emit = [&](int i, const float* tot) {
    const int u = u0 + i;
    bool valid;
    int li = -1;
    if (u < R) {
      valid = u < n_held && sHeld[u] != 0;
      sInv[i] = valid ? -2 : -1;  // -2: an attended held row
    } else {
      li = sInv[i];
      valid = li >= 0;
    }
#pragma unroll
    for (int g = 0; g < G; ++g) sA[g * chunk + i] = valid ? tot[g] * L.scale : kNegInf;
    if (policy && li >= 0) {
      // this CTA's block of the exchange, by physical row
      const float e = tot[G];
      sX[rank * gm.xs + i] = e;
      if (snap) {
        const float x = e * L.scale;
        if (x > em) {
          el = (em == kNegInf ? 0.f : el * __expf(em - x)) + 1.f;
          em = x;
        } else {
          el += __expf(x - em);
        }
      }
    }
  };
  // TMEM: the scoring tiles' accumulators, then (tensor-core P.V) the 16 columns of O^T
  uint32_t tbase = 0, tcols = 0;
  int colO = 0;
  if constexpr (MMA) {
    // tcgen05: one thread issues, per 128-row tile, D/16 MMAs of 128 x N8 x 16 into TMEM; warps
    // then read their lane quarter of each tile with tcgen05.ld
    const int ntiles = (nrows + 127) >> 7;
    const int need = gm.krows / 128 * N8;
    colO = need;
    const int want = need + (PVMMA ? N8 : 0);
    tcols = want <= 32 ? 32u : want <= 64 ? 64u : want <= 128 ? 128u : want <= 256 ? 256u : 512u;
    if (warp == 0) tmem_alloc(sTmem, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tbase = *sTmem;
    if (tid == 0 && ntiles > 0) {
      const uint32_t a0 = smem_u32(sK), b0 = smem_u32(sQb);
      for (int mt = 0; mt < ntiles; ++mt)
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t pl = ks >> 2, kin = ks & 3;
          const uint32_t aa = a0 + pl * (uint32_t)gm.krows * 128u + (uint32_t)mt * 128u * 128u + kin * 32u;
          const uint32_t bb = b0 + pl * (uint32_t)N8 * 128u + kin * 32u;
          umma_f16(tbase + (uint32_t)(mt * N8), umma_desc_k_sw128(aa), umma_desc_k_sw128(bb), kIdesc, ks > 0);
        }
      umma_commit(&bars[2]);
    }
    if (ntiles > 0 && !__syncthreads_and(mbar_wait(&bars[2], 0)) && tid == 0) set_status(st, HC_DEV_TIMEOUT);
    tc_fence_after();
    // warp w reads lane quarter w % 4 of tiles w / 4, w / 4 + 4, ...: rows 32 w + 512 k + lane;
    // with tensor-core P.V it also takes the maxima of its rows' attention logits
    float xm[G];
#pragma unroll
    for (int g = 0; g < G; ++g) xm[g] = kNegInf;
    for (int mt = warp >> 2; mt < ntiles; mt += kStepWarps / 4) {
      const int q4 = warp & 3;
      float v[NL];
#pragma unroll
      for (int c = 0; c < NL; c += 8) tmem_ld_x8(tbase + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(mt * N8 + c), v + c);
      const int i = mt * 128 + q4 * 32 + lane;
      if (i < nrows) {
        emit(i, v);
        if constexpr (PVMMA)
#pragma unroll
          for (int g = 0; g < G; ++g) xm[g] = fmaxf(xm[g], sA[g * chunk + i]);
      }
    }
    if constexpr (PVMMA) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        xm[g] = warp_max(xm[g]);
        if (lane == 0) sWst[warp * G + g] = xm[g];
      }
    }
    tc_fence_before();
    __syncthreads();
    if (!PVMMA && warp == 0) tmem_dealloc(tbase, tcols);
  } else
  {
    const int sub = lane & 7, tk = lane >> 3;
    float2 qr[QREG ? G + 1 : 1][QREG ? EPL / 2 : 1];
    if constexpr (QREG) {
#pragma unroll
      for (int g = 0; g <= G; ++g)
#pragma unroll
        for (int j = 0; j < CPL; ++j)
#pragma unroll
          for (int e = 0; e < VE / 2; ++e) {
            const int dd = (j * 8 + sub) * VE + 2 * e;
            qr[g][j * (VE / 2) + e] = make_float2(sQ[g * D + dd], sQ[g * D + dd + 1]);
          }
    }
    for (int base = warp * 4; base < nrows; base += 4 * kStepWarps) {
      const int i = base + tk;
      float2 acc[G + 1];
#pragma unroll
      for (int g = 0; g <= G; ++g) acc[g] = make_float2(0.f, 0.f);
      if (i < nrows) {
        const T* row = sK + (size_t)i * D;
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
          const int c = j * 8 + sub;
          float kf[VE];
          unpack16<DT>(*reinterpret_cast<const uint4*>(row + c * VE), kf);
#pragma unroll
          for (int g = 0; g <= G; ++g)
#pragma unroll
            for (int e = 0; e < VE / 2; ++e) {
              float2 q2;
              if constexpr (QREG) q2 = qr[g][j * (VE / 2) + e];
              else q2 = *reinterpret_cast<const float2*>(sQ + g * D + c * VE + 2 * e);
              acc[g] = __ffma2_rn(q2, make_float2(kf[2 * e], kf[2 * e + 1]), acc[g]);
            }
        }
      }
      float tot[G + 1];
#pragma unroll
      for (int g = 0; g <= G; ++g) {
        tot[g] = acc[g].x + acc[g].y;
        tot[g] += __shfl_xor_sync(0xffffffffu, tot[g], 4);
        tot[g] += __shfl_xor_sync(0xffffffffu, tot[g], 2);
        tot[g] += __shfl_xor_sync(0xffffffffu, tot[g], 1);
      }
      if (sub == 0 && i < nrows) emit(i, tot);
    }
  }
  // each warp's statistics partial into this CTA's block of the exchange, which goes to every
  // CTA of the cluster as one bulk copy each once the block is complete
  if (policy) {
    if (snap) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, em, o), l2 = __shfl_xor_sync(0xffffffffu, el, o);
        const float mx = fmaxf(em, m2);
        el = (em == kNegInf ? 0.f : el * __expf(em - mx)) + (m2 == kNegInf ? 0.f : l2 * __expf(m2 - mx));
        em = mx;
      }
      if (lane == 0) {
        sX[rank * gm.xs + chunk + 2 * warp] = em;
        sX[rank * gm.xs + chunk + 2 * warp + 1] = el;
      }
    }
    fence_proxy_async_smem();  // the bulk copies read the block through the async proxy
  }

  // ---- flash-decode partial of every warp over its rows -------------------------------------
  // warp w takes rows [w rpw, (w + 1) rpw) + k 16 rpw (rpw = ceil(nrows / 16), at most 32): the
  // rows are spread evenly over the warps whatever lane quarter of TMEM scored them
  const int rpw = min(32, (nrows + kStepWarps - 1) / kStepWarps);
  auto row_warp = [&](int i) { return (i / rpw) % kStepWarps; };
  // V rows landed (this barrier also publishes every warp's logits); the warp whose rows hold
  // the new slot puts the new value in place, each lane its own columns, the ones it reads
  if (!__syncthreads_and(mbar_wait(&bars[1], 0)) && tid == 0) set_status(st, HC_DEV_TIMEOUT);
  if (policy && warp == 1 && lane < ncta && lane != rank)
    bulk_s2cluster(sX + (size_t)rank * gm.xs, (uint32_t)gm.xs * 4u, &bars[4], (uint32_t)lane);
  constexpr int CW = D / 32;  // V columns per lane
  const int col0 = lane * CW;
  if constexpr (!PVMMA)
    if (i_new >= 0 && row_warp(i_new) == warp)
#pragma unroll
      for (int c = 0; c < CW; ++c) sV[(size_t)i_new * D + col0 + c] = sVn[col0 + c];
  // the K rows are no longer read: their area holds the warp partials [warp][G][D], the
  // probabilities of each warp's rows [warp][32][G] and the warps' (max, sum) [warp][G][2]
  float* red = reinterpret_cast<float*>(smem + M.k);
  float* sPw = red + (size_t)kStepWarps * G * D;
  float* sWml = sPw + (size_t)kStepWarps * 32 * G;
  float wm[G], wl[G];
  float2 acc[G][CW / 2];
  auto warp_partial = [&]() {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      wm[g] = kNegInf;
      wl[g] = 0.f;
#pragma unroll
      for (int c = 0; c < CW / 2; ++c) acc[g][c] = make_float2(0.f, 0.f);
    }
    for (int b = warp * rpw; b < nrows; b += kStepWarps * rpw)
      if (lane < rpw && b + lane < nrows)
#pragma unroll
        for (int g = 0; g < G; ++g) wm[g] = fmaxf(wm[g], sA[g * chunk + b + lane]);
#pragma unroll
    for (int g = 0; g < G; ++g) wm[g] = warp_max(wm[g]);
    float* pw = sPw + (size_t)warp * 32 * G;
    for (int b = warp * rpw; b < nrows; b += kStepWarps * rpw) {
      const int i = b + lane;
      const bool in = lane < rpw && i < nrows;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float x = in ? sA[g * chunk + i] : kNegInf;
        const float pr = x == kNegInf ? 0.f : __expf(x - wm[g]);
        pw[lane * G + g] = pr;
        wl[g] += pr;
      }
      // rows read: not a free slot or an unattended held row (their V is never read)
      const unsigned live = __ballot_sync(0xffffffffu, in && sInv[i] != -1);
      __syncwarp();
      const int nr = min(rpw, nrows - b);
#pragma unroll 4
      for (int r = 0; r < nr; ++r) {
        // branch-free: a row not read contributes p = 0 times v = 0 (its V may hold anything)
        const bool on = (live >> r) & 1u;
        float pv[G], vf[CW];
        if constexpr (G % 4 == 0) {
#pragma unroll
          for (int g = 0; g < G; g += 4) {
            const float4 t = reinterpret_cast<const float4*>(pw + r * G)[g / 4];
            pv[g] = t.x; pv[g + 1] = t.y; pv[g + 2] = t.z; pv[g + 3] = t.w;
          }
        } else if constexpr (G == 2) {
          const float2 t = *reinterpret_cast<const float2*>(pw + r * G);
          pv[0] = t.x; pv[1] = t.y;
        } else {
          pv[0] = pw[r];
        }
        unpack_n<DT, CW>(sV + (size_t)(b + r) * D + col0, vf);
#pragma unroll
        for (int c = 0; c < CW; ++c) vf[c] = on ? vf[c] : 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int c = 0; c < CW / 2; ++c)
            acc[g][c] = __ffma2_rn(make_float2(pv[g], pv[g]), make_float2(vf[2 * c], vf[2 * c + 1]), acc[g][c]);
      }
      __syncwarp();
    }
#pragma unroll
    for (int g = 0; g < G; ++g) wl[g] = warp_sum(wl[g]);
  };

  // ---- tensor-core P.V (16-bit, D = 128): the probabilities are the B operand (N8 query-head
  //      rows x rows of this part, K-major, 128-byte swizzle, in the K area), V^T the MN-major A
  //      operand straight from the TMA's planes, O^T (D lanes x N8 columns) accumulates in TMEM ---
  const int kext = PVMMA ? (nrows + 15) & ~15 : 0;  // rows the MMAs reduce over, 16 per instruction
  unsigned char* sPo = smem + M.k;
  unsigned char* sVb = reinterpret_cast<unsigned char*>(sV);
  float mg[G];
  uint32_t pv_phase = 0;
  // remax: take the maxima again from the logits (after rows left the attention)
  auto build_pv = [&](bool remax) {
    if (remax) {
      float xm[G];
#pragma unroll
      for (int g = 0; g < G; ++g) xm[g] = kNegInf;
      for (int i = tid; i < nrows; i += kStepThreads)
#pragma unroll
        for (int g = 0; g < G; ++g) xm[g] = fmaxf(xm[g], sA[g * chunk + i]);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        xm[g] = warp_max(xm[g]);
        if (lane == 0) sWst[warp * G + g] = xm[g];
      }
      __syncthreads();
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float m = kNegInf;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) m = fmaxf(m, sWst[w * G + g]);
      mg[g] = m;
    }
    float ls[G];
#pragma unroll
    for (int g = 0; g < G; ++g) ls[g] = 0.f;
    for (int i = tid; i < kext; i += kStepThreads) {
      const bool att = i < nrows && sInv[i] != -1;
      const int c = (i & 63) >> 3;
      unsigned char* prow = sPo + (size_t)(i >> 6) * (N8 * 128) + (i & 7) * 2;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float x = att ? sA[g * chunk + i] : kNegInf;
        const float pr = x == kNegInf ? 0.f : __expf(x - mg[g]);
        ls[g] += pr;
        *reinterpret_cast<T*>(prow + (size_t)g * 128 + ((c ^ (g & 7)) << 4)) = E::from_f(pr);
      }
      if (!att)  // a row not attended: its V may hold anything, and the MMA multiplies it by 0
#pragma unroll
        for (int pl = 0; pl < PL; ++pl)
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<uint4*>(sVb + (size_t)pl * gm.vrows * 128 + (size_t)i * 128)[q] = make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      ls[g] = warp_sum(ls[g]);
      if (lane == 0) sWst[kStepWarps * G + warp * G + g] = ls[g];
    }
    fence_proxy_async_smem();  // generic writes above are read by the tensor cores
    __syncthreads();
    if (tid == kStepThreads - 32 && kext > 0) {  // a thread of the last warp, which ranks the fewest tokens
      tc_fence_after();
      constexpr uint32_t idesc = kIdesc | (1u << 15);  // A (V^T) MN-major
      const uint32_t a0 = smem_u32(sVb), b0 = smem_u32(sPo), lbo = (uint32_t)gm.vrows * 128u;
      for (int ks = 0; ks < kext / 16; ++ks) {
        const uint32_t aa = a0 + (uint32_t)ks * 2048u;
        const uint32_t bb = b0 + (uint32_t)(ks >> 2) * (N8 * 128u) + (uint32_t)(ks & 3) * 32u;
        umma_f16(tbase + (uint32_t)colO, umma_desc_mn_sw128(aa, lbo), umma_desc_k_sw128(bb), idesc, ks > 0);
      }
      umma_commit(&bars[3]);
    }
  };
  if constexpr (PVMMA) {
    // the new value into its swizzled row, before the MMAs read V
    if (i_new >= 0 && tid < D) {
      const int c = (tid & 63) >> 3;
      *reinterpret_cast<T*>(sVb + (size_t)(tid >> 6) * gm.vrows * 128 + (size_t)i_new * 128 + ((c ^ (i_new & 7)) << 4) +
                            (tid & 7) * 2) = sVn[tid];
    }
    build_pv(false);
  } else {
    warp_partial();
  }
  float pe[G];      // probabilities of the evicted row, when its term is subtracted
  int fix_ev = -1;  // that row (tensor-core P.V)

  // ---- policy: every CTA holds every head's eviction logits and statistics partials and ranks
  //      the prefix itself, so every CTA makes the same selection -----------------------------
  int n_ev = 0;
  int ev_slot = -1, ev_dst = -1, ev_li = -1;  // the single evicted token, when exactly one leaves
  if (policy) {
    if (!mbar_wait(&bars[4], 0)) set_status(st, HC_DEV_TIMEOUT);  // every other CTA's block landed
    float* sC = sRed;  // per head: the softmax max and the reciprocal of the sum
    if (snap) {
      // each head's statistics over its S hot tokens from its P CTAs' warp partials
      if (warp < L.Hk) {
        const int np = P * kStepWarps;
        float m = kNegInf, l = 0.f;
        for (int j = lane; j < np; j += 32) {
          const int r2 = warp * P + j / kStepWarps, w = j % kStepWarps;
          const float* st2 = sX + (size_t)r2 * gm.xs + chunk + 2 * w;
          const float m2 = st2[0], l2 = st2[1];
          const float mx = fmaxf(m, m2);
          l = (m == kNegInf ? 0.f : l * __expf(m - mx)) + (m2 == kNegInf ? 0.f : l2 * __expf(m2 - mx));
          m = mx;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
          const float mx = fmaxf(m, m2);
          l = (m == kNegInf ? 0.f : l * __expf(m - mx)) + (m2 == kNegInf ? 0.f : l2 * __expf(m2 - mx));
          m = mx;
        }
        if (lane == 0) {
          sC[2 * warp] = m;
          sC[2 * warp + 1] = 1.f / l;
        }
      }
      __syncthreads();
    }
    // the key of prefix token li. SnapKV (scoring.py:72-78): the max-pooled probability is
    // exp(max logit - M) / L, exp and the division being monotone; hot/cold (cache.py:68-69): the
    // raw logit / sqrt(D). Then the mean over heads.
    const int pad = L.pool_kernel > 1 ? L.pool_kernel / 2 : 0;
    const bool pmax = L.pooling == HC_POOL_MAX;
    const float inv = 1.f / sqrtf((float)L.D);
    // head hh's logit of token u: sX[hh * P * xs + sLoc[u]] (the part and row of u's slot)
    const int hstride = P * gm.xs;
    auto token_key = [&](int li) {
      const int ua = max(0, li - pad), ub = min(S - 1, li + pad);
      float v = 0.f;
      if (snap && pmax && pad == 3) {
        // the configured 7-wide max pool: indices clamped into [0, S), repeats leave the max alone
        int uu[7];
#pragma unroll
        for (int k = 0; k < 7; ++k) uu[k] = sLoc[min(max(li - 3 + k, 0), S - 1)];
#pragma unroll 4
        for (int hh = 0; hh < L.Hk; ++hh) {
          const float* x = sX + (size_t)hh * hstride;
          float mx = x[uu[0]];
#pragma unroll
          for (int k = 1; k < 7; ++k) mx = fmaxf(mx, x[uu[k]]);
          v += __expf(mx * L.scale - sC[2 * hh]) * sC[2 * hh + 1];
        }
        return fkey(v / (float)L.Hk);
      }
      for (int hh = 0; hh < L.Hk; ++hh) {
        const float* x = sX + (size_t)hh * hstride;
        float t;
        if (snap) {
          const float mh = sC[2 * hh], rl = sC[2 * hh + 1];
          if (pad == 0 || pmax) {
            float mx = kNegInf;
            for (int u = ua; u <= ub; ++u) mx = fmaxf(mx, x[sLoc[u]]);
            t = __expf(mx * L.scale - mh) * rl;
          } else {
            t = 0.f;
            for (int u = ua; u <= ub; ++u) t += __expf(x[sLoc[u]] * L.scale - mh) * rl;
            t /= (float)L.pool_kernel;
          }
        } else {
          t = x[sLoc[li]] * inv;
        }
        v += t;
      }
      return fkey(v / (float)L.Hk);
    };
    n_ev = n_ev_plan;
    if (n_ev == 1) {
      // one token leaves: the lowest key, equal keys evict the higher index
      unsigned long long best = ~0ull;
      for (int li = tid; li < pl.prefix; li += kStepThreads) {
        const unsigned long long c = ((unsigned long long)token_key(li) << 32) | (0xffffffffu - (uint32_t)li);
        best = c < best ? c : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
        best = y < best ? y : best;
      }
      unsigned long long* sBest = reinterpret_cast<unsigned long long*>(sRed + 96);  // per warp
      if (lane == 0) sBest[warp] = best;
      __syncthreads();
      best = sBest[0];
#pragma unroll
      for (int w = 1; w < kStepWarps; ++w) best = sBest[w] < best ? sBest[w] : best;
      const int li_ev = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffu));
      ev_slot = phys_of(li_ev);
      ev_li = li_ev;
      ev_dst = cold_head + cold_count;  // cold_head < ccap and cold_count <= ccap
      if (ev_dst >= d.ccap) ev_dst -= d.ccap;
      if (d.ccap <= 0) ev_dst = -1;
      // warm L2 for the copies into the cold ring done at the end of the kernel
      if (ev_slot >= 0 && ev_slot < cap) {
        constexpr int LPR = ROWB / 128;  // 128-byte lines per row
        if (p == 0 && tid < 2 * LPR) {
          const char* src = reinterpret_cast<const char*>(tid & 1 ? d.hot_v : d.hot_kpre);
          prefetch_l2(src + ((size_t)h * cap + ev_slot) * ROWB + (tid >> 1) * 128);
        }
        if (rank == ncta - 1 && tid < L.Hk * LPR)
          prefetch_l2(reinterpret_cast<const char*>(d.hot_kpre) + ((size_t)(tid / LPR) * cap + ev_slot) * ROWB +
                      (tid % LPR) * 128);
      }
      // compaction of own words: entries after li_ev move down by one
      for (int i = tid; i < own_n; i += kStepThreads) {
        const int li = own0 + i;
        const int ph = phys_of(li);
        if (li > li_ev) d.hot_ord[li - 1] = ph;
        else if (li == li_ev && n_free - 1 < cap) d.hot_free[n_free - 1] = ph;
      }
      // the evicted row leaves the attention partial that holds it: its term is subtracted, or,
      // where that row carried most of a head's mass (the difference would cancel), the partial
      // is recomputed without it
      const int i_ev = row_of_slot(ev_slot);
      if constexpr (PVMMA) {
        if (i_ev >= 0) {  // the same in every thread of the CTA
          bool redo = false;
#pragma unroll
          for (int g = 0; g < G; ++g) {
            float l = 0.f;
#pragma unroll
            for (int w = 0; w < kStepWarps; ++w) l += sWst[kStepWarps * G + w * G + g];
            const float x = sA[g * chunk + i_ev];
            pe[g] = x == kNegInf ? 0.f : __expf(x - mg[g]);
            redo |= !(l - pe[g] >= 0.25f * l);
          }
          if (redo) {
            // the first MMAs read the operands until they complete
            if (!__syncthreads_and(mbar_wait(&bars[3], 0)) && tid == 0) set_status(st, HC_DEV_TIMEOUT);
            if (tid < G) sA[tid * chunk + i_ev] = kNegInf;
            __syncthreads();
            build_pv(true);
            pv_phase = 1;
          } else {
            fix_ev = i_ev;
          }
        }
      } else if (i_ev >= 0 && row_warp(i_ev) == warp) {
        bool redo = false;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float x = sA[g * chunk + i_ev];
          pe[g] = x == kNegInf ? 0.f : __expf(x - wm[g]);
          redo |= !(wl[g] - pe[g] >= 0.25f * wl[g]);
        }
        if (redo) {
          if (lane < G) sA[lane * chunk + i_ev] = kNegInf;
          __syncwarp();
          warp_partial();
        } else {
          float vf[CW];
          unpack_n<DT, CW>(sV + (size_t)i_ev * D + col0, vf);
#pragma unroll
          for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int c = 0; c < CW / 2; ++c)
              acc[g][c] = __ffma2_rn(make_float2(-pe[g], -pe[g]), make_float2(vf[2 * c], vf[2 * c + 1]), acc[g][c]);
            wl[g] -= pe[g];
          }
        }
      }
    } else {
      // every CTA needs every prefix key: own keys to all CTAs (barrier C)
      const int own_p = max(0, min(own_n, pl.prefix - own0));  // this CTA's own prefix tokens
      for (int li = own0 + tid; li < own0 + own_p; li += kStepThreads) sKey[li] = token_key(li);
      __syncthreads();
      for (int k = tid; k < ncta * own_p; k += kStepThreads) {
        const int r2 = k / own_p, li = own0 + (k - r2 * own_p);
        if (r2 != rank) cluster.map_shared_rank(sKey, r2)[li] = sKey[li];
      }
      cluster.sync();
      // rank every prefix token against all prefix keys: kept when fewer than n_top keys are
      // above it (equal keys: the lower index ranks above); one word of 32 tokens per warp pass
      for (int wi = warp; wi < nwords; wi += kStepWarps) {
        const int t = wi * 32 + lane;
        bool keep = t < S;
        if (t < pl.prefix) {
          const uint32_t kt = sKey[t];
          int cnt = 0;
#pragma unroll 4
          for (int u = 0; u < pl.prefix; ++u) {
            const uint32_t ku = sKey[u];
            cnt += (ku > kt) || (ku == kt && u < t);
          }
          keep = cnt < pl.ntop;
        }
        const unsigned evw = __ballot_sync(0xffffffffu, t < S && !keep);
        if (lane == 0) sMask[wi] = evw;
      }
      __syncthreads();
      // kept and evicted tokens before this CTA's words, and all evicted
      int kb = 0, eb = 0, tot_ev = 0;
      for (int w = 0; w < nwords; ++w) {
        const uint32_t inw = (w < nwords - 1 || (S & 31) == 0) ? 0xffffffffu : ((1u << (S & 31)) - 1u);
        const uint32_t evw = sMask[w];
        tot_ev += __popc(evw);
        if (w < w0) {
          kb += __popc(inw & ~evw);
          eb += __popc(evw);
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
          const unsigned km = __ballot_sync(0xffffffffu, keep), em2 = __ballot_sync(0xffffffffu, ev);
          const int ph = in ? phys_of(t) : -1;
          if (keep) d.hot_ord[kb + __popc(km & lt)] = ph;
          if (ev) {
            const int j = eb + __popc(em2 & lt), jl = nloc + __popc(em2 & lt);
            if (n_free - 1 + j < cap) d.hot_free[n_free - 1 + j] = ph;
            sEvl[3 * jl] = ph;
            sEvl[3 * jl + 1] = (j >= n_ev - d.ccap) ? (int)(((long)cold_head + cold_count + j) % d.ccap) : -1;
            sEvl[3 * jl + 2] = t;
          }
          kb += __popc(km);
          eb += __popc(em2);
          nloc += __popc(em2);
        }
        if (lane == 0) sMisc[4] = nloc;
      }
      // the evicted rows leave the attention: the partials are recomputed
      for (int i = tid; i < nrows; i += kStepThreads) {
        const int li = sInv[i];
        if (li >= 0 && ((sMask[li >> 5] >> (li & 31)) & 1u))
#pragma unroll
          for (int g = 0; g < G; ++g) sA[g * chunk + i] = kNegInf;
      }
      if constexpr (PVMMA) {
        // the first MMAs read the operands until they complete
        if (kext > 0 && !__syncthreads_and(mbar_wait(&bars[3], 0)) && tid == 0) set_status(st, HC_DEV_TIMEOUT);
        __syncthreads();
        build_pv(true);
        pv_phase = 1;
      } else {
        __syncthreads();
        warp_partial();
      }
    }
  }

  // ---- the part's partial per column, each column block sent to the CTA of head h that
  //      finalizes it ---------------------------------------------------------------------------
  const int DB = D / P;
  if constexpr (PVMMA) {
    // warps 0-3 read O^T from TMEM (lane = column d, column g = query head), subtract the evicted
    // row's term where it is taken out here, and send
    float lg[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) l += sWst[kStepWarps * G + w * G + g];
      lg[g] = fix_ev >= 0 ? l - pe[g] : l;
    }
    if (warp < 4) {
      float o[8];
      if (kext > 0) {
        if (!mbar_wait(&bars[3], pv_phase)) set_status(st, HC_DEV_TIMEOUT);
        tc_fence_after();
        tmem_ld_x8(tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)colO, o);
      } else {
#pragma unroll
        for (int g = 0; g < 8; ++g) o[g] = 0.f;
      }
      const int dd = warp * 32 + lane;
      if (fix_ev >= 0) {
        const int c = (dd & 63) >> 3;
        const float ve = E::to_f(*reinterpret_cast<const T*>(sVb + (size_t)(dd >> 6) * gm.vrows * 128 +
                                                             (size_t)fix_ev * 128 + ((c ^ (fix_ev & 7)) << 4) + (dd & 7) * 2));
#pragma unroll
        for (int g = 0; g < G; ++g) o[g] = fmaf(-E::round(pe[g]), ve, o[g]);
      }
      const int q = dd / DB, col = dd - q * DB;
      float* dst = q == p ? sO : cluster.map_shared_rank(sO, h * P + q);
#pragma unroll
      for (int g = 0; g < G; ++g) dst[((size_t)p * G + g) * DB + col] = o[g];
      if (col == 0) {
        float* dml = q == p ? sML : cluster.map_shared_rank(sML, h * P + q);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          dml[2 * (p * G + g)] = mg[g];
          dml[2 * (p * G + g) + 1] = lg[g];
        }
      }
    }
    tc_fence_before();
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float* dst = red + ((size_t)warp * G + g) * D + col0;
      if constexpr (CW % 4 == 0) {
#pragma unroll
        for (int c = 0; c < CW / 2; c += 2)
          reinterpret_cast<float4*>(dst)[c / 2] = make_float4(acc[g][c].x, acc[g][c].y, acc[g][c + 1].x, acc[g][c + 1].y);
      } else {
#pragma unroll
        for (int c = 0; c < CW / 2; ++c) reinterpret_cast<float2*>(dst)[c] = acc[g][c];
      }
    }
    if (lane == 0)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        sWml[2 * (warp * G + g)] = wm[g];
        sWml[2 * (warp * G + g) + 1] = wl[g];
      }
    __syncthreads();
    for (int k = tid; k < G * D; k += kStepThreads) {
      const int g = k / D, dd = k - g * D;
      float Mx = kNegInf;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) Mx = fmaxf(Mx, sWml[2 * (w * G + g)]);
      float v = 0.f, l = 0.f;
#pragma unroll
      for (int w = 0; w < kStepWarps; ++w) {
        const float mw = sWml[2 * (w * G + g)];
        const float e = mw == kNegInf ? 0.f : __expf(mw - Mx);
        v = fmaf(red[((size_t)w * G + g) * D + dd], e, v);
        l = fmaf(sWml[2 * (w * G + g) + 1], e, l);
      }
      const int q = dd / DB, col = dd - q * DB;
      float* dst = q == p ? sO : cluster.map_shared_rank(sO, h * P + q);
      dst[((size_t)p * G + g) * DB + col] = v;
      if (col == 0) {
        float* dml = q == p ? sML : cluster.map_shared_rank(sML, h * P + q);
        dml[2 * (p * G + g)] = Mx;
        dml[2 * (p * G + g) + 1] = l;
      }
    }
  }
  cluster.sync();  // last barrier: no distributed shared memory access after this point
  if (PVMMA && warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, tcols);
  }
  T* outp = reinterpret_cast<T*>(a.out) + ((size_t)s * L.Hq + (size_t)h * G) * D + (size_t)p * DB;
  for (int k = tid; k < G * DB; k += kStepThreads) {
    const int g = k / DB, col = k - g * DB;
    float Mx = kNegInf;
    for (int q = 0; q < P; ++q) Mx = fmaxf(Mx, sML[2 * (q * G + g)]);
    float Ls = 0.f, Os = 0.f;
    for (int q = 0; q < P; ++q) {
      const float w = __expf(sML[2 * (q * G + g)] - Mx);
      Ls = fmaf(sML[2 * (q * G + g) + 1], w, Ls);
      Os = fmaf(sO[((size_t)q * G + g) * DB + col], w, Os);
    }
    float r = Os / Ls;
    if (a.overflow_nan && Mx >= kExpOverflow) r = __int_as_float(0x7fc00000);
    outp[(size_t)g * D + col] = E::from_f(r);
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
  // ---- work nothing in this kernel waits for: evicted payloads into the cold ring -----------
  if (n_ev == 1) {
    // spread over the cluster: the first CTA of each head copies that head's rows, the last
    // CTA writes the index vector and the position
    if (ev_dst >= 0 && ev_slot >= 0 && ev_slot < cap) {
      if (p == 0 && warp == 0) {
        const size_t roff = ((size_t)h * cap + ev_slot) * D;
        const size_t doff = ((size_t)ev_dst * L.Hk + h) * D;
        for (int c = lane; c < KCH; c += 32) {
          reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.cold_kpre) + doff)[c] =
              reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(d.hot_kpre) + roff)[c];
          reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.cold_v) + doff)[c] =
              reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(d.hot_v) + roff)[c];
        }
      }
      if (rank == ncta - 1 && warp == kStepWarps - 1) {
        const int64_t pv = ev_li == n_hot ? cur_pos : d.hot_pos[ev_slot];
        step_evict_vec<DT, D>(L, d, ev_slot, ev_dst, pv);
      }
    } else if (ev_dst >= 0 && rank == 0 && tid == 0) {
      set_status(st, HC_DEV_INDEX);
    }
  } else if (n_ev > 1) {
    const int nloc = sMisc[4];
    for (int q = warp; q < nloc; q += kStepWarps) {
      const int slot = sEvl[3 * q], dst = sEvl[3 * q + 1], li = sEvl[3 * q + 2];
      if (dst < 0) continue;  // more tokens evicted than the ring holds: the oldest are dropped
      const int64_t pv = li == n_hot ? cur_pos : (slot >= 0 && slot < cap ? d.hot_pos[slot] : -1);
      step_evict_one<DT, D>(L, d, slot, dst, pv);
    }
  }
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
int step_parts(int Hk) { return (Hk >= 1 && Hk <= kStepMaxCluster && kStepMaxCluster % Hk == 0) ? kStepMaxCluster / Hk : 0; }

static StepGeom layer_geom(const hc_layer& L, int use_held) {
  return step_geom(L.Hk, L.max_cap, L.max_r, use_held, L.dtype != HC_F32, L.dtype != HC_F32 && L.D == 128);
}

size_t step_smem_bytes(const hc_layer& L, int use_held) {
  const StepGeom g = layer_geom(L, use_held);
  if (!g.P || L.Hq % L.Hk) return 0;
  const int esz = L.dtype == HC_F32 ? 4 : 2;
  const int G = L.Hq / L.Hk;
  if (G > 8 || (L.D * esz) % 128 || L.D % g.P) return 0;
  return step_smem(L.D, esz, G, L.Hk, L.max_r, g).total;
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
static cudaError_t step_t(const StepArgs& a, cudaStream_t stream, bool check_only) {
  using T = typename Elem<DT>::T;
  const StepSmem M = step_smem(D, sizeof(T), G, a.L.Hk, a.L.max_r, a.g);
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
  if (e != cudaSuccess || check_only) return e;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int DT, int D>
static cudaError_t step_g(const StepArgs& a, cudaStream_t stream, bool check_only) {
  switch (a.L.Hq / a.L.Hk) {
    case 1: return step_t<DT, D, 1>(a, stream, check_only);
    case 2: return step_t<DT, D, 2>(a, stream, check_only);
    case 4: return step_t<DT, D, 4>(a, stream, check_only);
    case 8: return step_t<DT, D, 8>(a, stream, check_only);
  }
  return cudaErrorNotSupported;
}

cudaError_t launch_step(const hc_layer& L, const void* q, int64_t qss, const void* k, const void* v, int64_t kvss,
                        const void* c, const void* sn, const int64_t* pos, int use_held, void* out, int overflow_nan,
                        int early, cudaStream_t stream, bool check_only) {
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
  a.early = early & (HC_STEP_EARLY_HOT | HC_STEP_EARLY_HELD);
  a.g = layer_geom(L, use_held);
  if (L.dtype == HC_F32 && L.D == 128) return step_g<HC_F32, 128>(a, stream, check_only);
  if (L.dtype == HC_F16 && L.D == 128) return step_g<HC_F16, 128>(a, stream, check_only);
  if (L.dtype == HC_BF16 && L.D == 128) return step_g<HC_BF16, 128>(a, stream, check_only);
  if (L.dtype == HC_F32 && L.D == 64) return step_g<HC_F32, 64>(a, stream, check_only);
  if (L.dtype == HC_F16 && L.D == 64) return step_g<HC_F16, 64>(a, stream, check_only);
  if (L.dtype == HC_BF16 && L.D == 64) return step_g<HC_BF16, 64>(a, stream, check_only);
  return cudaErrorNotSupported;
}

}  // namespace hc
