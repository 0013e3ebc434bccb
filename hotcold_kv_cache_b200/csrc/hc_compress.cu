// Hot-tier compression with eviction into the cold ring.
//
// Reference flow (HotColdLayer._compress_if_needed, cache.py:37-128): score every hot
// token, keep the top-n_top of the prefix plus the recent tail, gather the kept tokens,
// copy the evicted ones to pinned host memory, and hand them to the cold store, which
// builds one index vector per token in a Python loop (controller.py:190-238). Under
// HC_POLICY_SNAPKV the score is SnapKV's importance (scoring.py:50-79) averaged over KV
// heads and the keep set follows keep_index (scoring.py:110-132).
//
// Here the whole flow stays in HBM:
//   score_kernel   (seq, KV head, token chunk): bulk-copies the chunk's post-RoPE keys to
//                  shared memory and scores them against the GQA-mean observation queries;
//                  hot/cold: one logit sum per token; SnapKV: one logit per (row, token)
//                  plus the chunk's softmax partials per row.
//   stats/token    (large inputs only) SnapKV softmax statistics per row, then per-token
//                  importance, pooling and the mean over KV heads.
//   select_kernel  (one CTA per sequence): exact top-k of the prefix (ties to the lower
//                  index), order-preserving compaction of the logical order, free-slot
//                  push, ring plan; small evictions are copied inline.
//   select_cluster_kernel  (prompts; a cluster of up to 16 CTAs per sequence): the same top-k
//                  and keep / evict lists, the histograms of the radix passes summed through
//                  distributed shared memory; up to 16k tokens it also computes the token
//                  scores (no token_kernel).
//   evict_kernel   (large evictions / prompt): payload copies into the cold ring with the
//                  index vector (mean over KV heads of the pre-RoPE key, pad/crop,
//                  L2-normalise; controller.py:178-182) and, for a prompt, the kept
//                  tokens into the slab.
// Scores are float32 throughout (the reference rounds its GPU logits to the model dtype).

#include "hc_internal.cuh"
#include "hc_topk.cuh"

namespace hc {

constexpr int kScoreCH = 64;        // tokens per score CTA
constexpr int kInlineEvict = 32;    // evictions copied by the select CTA itself
constexpr size_t kSelectSmemMax = 200 * 1024;  // shared memory of the selection CTA's small path


// cache.py:44-53 (hot/cold) or scoring.py:117-120 with the trigger of cache.py:44 (SnapKV).
__device__ __forceinline__ Plan make_plan(const hc_layer& L, int budget, int S) {
  Plan p{S, 0, 0, 0, 0};
  if (S <= budget) return p;
  if (L.policy == HC_POLICY_HOTCOLD) {
    const int recent = min(min(L.recent, budget), S);
    const int prefix = S - recent;
    if (prefix <= 0) return p;
    int ntop = (int)((double)budget * L.topk_ratio);
    ntop = max(1, min(ntop, prefix));
    p = Plan{S, prefix, ntop, recent, 1};
  } else {
    const int window = min(L.recent, S);
    const int prefix = S - window;
    const int ntop = max(0, min(budget - window, prefix));
    p = Plan{S, prefix, ntop, window, 1};
  }
  return p;
}

struct CompressArgs {
  hc_layer L;
  const void* q_obs;
  int64_t qs_seq, qs_head, qs_tok;
  int tq;        // query rows provided
  int S_dense;   // prompt length (dense mode)
  int S_max;     // row stride of the per-token scratch arrays
  int max_chunks;
  const void* src_k;
  const void* src_v;
  const void* src_kpre;
  int64_t ss_seq, ss_head, ss_tok;
  const int64_t* src_pos;
  // scratch
  int* hdr;        // [n_seq][16]: S, prefix, ntop, nobs, active, n_keep_copy, n_evict, tq_used
  float* logits;   // [n_seq][Hk][tqmax][S_max]   (hot/cold: [n_seq][Hk][S_max])
  float* part;     // [n_seq][Hk][tqmax][max_chunks][2]
  float* stats;    // [n_seq][Hk][tqmax][2]
  float* imp;      // [n_seq][Hk][S_max]
  float* tok;      // [n_seq][S_max]
  uint8_t* sel;    // [n_seq][S_max]
  int* keep_src;   // [n_seq][S_max]
  int* ev_src;     // [n_seq][S_max]
  int* ev_dst;     // [n_seq][S_max]
  void* qb;        // [n_seq][Hk][32][D] GQA-mean observation rows in the model dtype (tensor-core path)
  int tqmax;
  int chunk_len;   // tokens per softmax partial in `part`
  int vec_ok;      // source rows and strides allow 16-byte copies (evict_kernel)
};

template <bool DENSE>
__device__ __forceinline__ int seq_len(const CompressArgs& a, const hc_seq_desc& d) {
  if constexpr (DENSE) return a.S_dense;
  return d.st->n_hot;
}

// ------------------------------------------------------------------------------------------
// score
// ------------------------------------------------------------------------------------------
template <int DT, int D, bool DENSE>
__global__ void __launch_bounds__(128) score_kernel(CompressArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int CH = kScoreCH;
  constexpr int ROWB = D * sizeof(T);
  constexpr int VEC = 16 / sizeof(T);
  constexpr int NJ = D / (8 * VEC);
  extern __shared__ __align__(128) unsigned char smem[];
  T* sK = reinterpret_cast<T*>(smem);
  float* sQ = reinterpret_cast<float*>(smem + sizeof(T) * CH * D);      // [tqmax + 1][D]
  float* sL = sQ + (size_t)(a.tqmax + 1) * D;                             // [tqmax][CH]
  const T** sRowp = reinterpret_cast<const T**>(sL + (size_t)a.tqmax * CH + 4);  // [CH] row sources
  constexpr int CPR = D / VEC;  // 16-byte chunks per row

  const int c = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const hc_layer& L = a.L;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  if (!pl.active) return;
  const int S = pl.S;
  if (c * CH >= S) return;
  const int t0 = c * CH, nt = min(CH, S - t0);
  const int tqu = min(pl.nobs, a.tq);
  const int G = L.Hq / L.Hk;

  // key rows of this chunk, gathered with 16-byte cp.async (an out-of-range slot is reported
  // and read as zeros)
  const T* row = nullptr;
  if (tid < nt) {
    const int t = t0 + tid;
    if constexpr (DENSE) {
      row = reinterpret_cast<const T*>(a.src_k) + (size_t)s * a.ss_seq + (size_t)h * a.ss_head + (size_t)t * a.ss_tok;
    } else {
      const int slot = d.hot_ord[t];
      if (slot >= 0 && slot < d.cap) row = reinterpret_cast<const T*>(d.hot_k) + ((size_t)h * d.cap + slot) * D;
      else set_status(d.st, HC_DEV_INDEX);
    }
  }
  if (tid < CH) sRowp[tid] = row;
  __syncthreads();
  for (int k = tid; k < nt * CPR; k += 128) {
    const int r = k / CPR, q = k % CPR;
    const T* src = sRowp[r];
    cp_async16(sK + (size_t)r * D + q * VEC, src ? src + q * VEC : reinterpret_cast<const T*>(a.q_obs), src ? 16 : 0);
  }
  cp_async_commit();
  // GQA-mean observation rows (cache.py:60-64 / scoring.py:17-26), rounded to the dtype
  const T* q = reinterpret_cast<const T*>(a.q_obs) + (size_t)s * a.qs_seq;
  for (int i = tid; i < tqu * D; i += 128) {
    const int r = i / D, dd = i % D;
    const int row = a.tq - tqu + r;
    float acc = 0.f;
    for (int g = 0; g < G; ++g)
      acc += E::to_f(q[(size_t)(h * G + g) * a.qs_head + (size_t)row * a.qs_tok + dd]);
    sQ[i] = E::round(acc / (float)G);
  }
  __syncthreads();
  const bool hotcold = L.policy == HC_POLICY_HOTCOLD;
  if (hotcold && tid < D) {  // logits are linear in q: sum the rows first
    float acc = 0.f;
    for (int r = 0; r < tqu; ++r) acc += sQ[r * D + tid];
    sQ[(size_t)a.tqmax * D + tid] = acc;  // the extra row holds the sum
  }
  cp_async_wait<0>();
  __syncthreads();

  const int sub = lane & 7, tk = lane >> 3;
  const int nrows = hotcold ? 1 : tqu;
  const float* qrows = hotcold ? sQ + (size_t)a.tqmax * D : sQ;
  for (int base = warp * 4; base < nt; base += 16) {
    const int t = base + tk;
    float kf[NJ * VEC];
    if (t < nt) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        uint4 u = *reinterpret_cast<const uint4*>(sK + (size_t)t * D + j * 8 * VEC + sub * VEC);
        unpack16<DT>(u, kf + j * VEC);
      }
    } else {
#pragma unroll
      for (int e = 0; e < NJ * VEC; ++e) kf[e] = 0.f;
    }
    for (int r = 0; r < nrows; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc = fmaf(qrows[r * D + j * 8 * VEC + sub * VEC + e], kf[j * VEC + e], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (sub == 0 && t < nt) {
        if (hotcold) {
          a.logits[((size_t)s * L.Hk + h) * a.S_max + t0 + t] = acc;
        } else {
          const int tg = t0 + t;
          // observation row r sits at index S - tqu + r; later keys are masked (scoring.py:72-74)
          const float x = (tg > S - tqu + r) ? kNegInf : acc * L.scale;
          sL[r * CH + t] = x;
          a.logits[(((size_t)s * L.Hk + h) * a.tqmax + r) * a.S_max + tg] = x;
        }
      }
    }
  }
  if (hotcold) return;
  __syncthreads();
  // chunk softmax partials per observation row
  for (int r = warp; r < tqu; r += 4) {
    float m = kNegInf;
    for (int t = lane; t < nt; t += 32) m = fmaxf(m, sL[r * CH + t]);
    m = warp_max(m);
    float l = 0.f;
    for (int t = lane; t < nt; t += 32) {
      const float x = sL[r * CH + t];
      l += (x == kNegInf) ? 0.f : __expf(x - m);
    }
    l = warp_sum(l);
    if (lane == 0) {
      float* p = a.part + ((((size_t)s * L.Hk + h) * a.tqmax + r) * a.max_chunks + c) * 2;
      p[0] = m;
      p[1] = l;
    }
  }
}

// ------------------------------------------------------------------------------------------
// SnapKV scoring on the 5th-generation tensor cores (16-bit dtypes, large inputs)
// ------------------------------------------------------------------------------------------
// The observation-window x prefix product (scoring.py:71-77) is a dense contraction per KV
// head: logits[t][r] = k_t . qbar_r * scale for 128-token tiles. snap_qbar_kernel writes the
// GQA-mean observation rows once; snap_tile_kernel gathers a tile of keys into the 128-byte
// swizzled K-major layout (cp.async), issues D/16 tcgen05.mma (M = 128 tokens, N = the rows
// padded to 16/32) into TMEM and reads one token per thread back with tcgen05.ld. Pass 0
// writes per-warp (32-token) softmax partials of every row; after stats_kernel, pass 1
// recomputes the tile and writes each token's importance sum_r softmax_r[t] directly, so the
// [rows][S] logits never go to HBM.
constexpr int kSnapTile = 128;

template <int DT, int D, bool DENSE>
__global__ void snap_qbar_kernel(CompressArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  const int h = blockIdx.x, s = blockIdx.z, r0 = blockIdx.y * 2;
  const hc_layer& L = a.L;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  const int tqu = pl.active ? min(min(pl.nobs, a.tq), 32) : 0;
  const int G = L.Hq / L.Hk;
  const T* q = reinterpret_cast<const T*>(a.q_obs) + (size_t)s * a.qs_seq;
  T* out = reinterpret_cast<T*>(a.qb) + ((size_t)s * L.Hk + h) * 32 * D;
  for (int i = r0 * D + threadIdx.x; i < (r0 + 2) * D; i += blockDim.x) {
    const int r = i / D, dd = i % D;
    float v = 0.f;
    if (r < tqu) {
      const int row = a.tq - tqu + r;
      float acc = 0.f;
      for (int g = 0; g < G; ++g) acc += E::to_f(q[(size_t)(h * G + g) * a.qs_head + (size_t)row * a.qs_tok + dd]);
      v = acc / (float)G;
    }
    out[i] = E::from_f(v);  // the dtype rounding of cache.py:60-64 / scoring.py:17-26
  }
}

// CTA (x, h, s) takes `tpc` consecutive tiles; the keys of tile i + 1 are gathered (cp.async,
// second buffer) while tile i is multiplied and its epilogue runs. Shared memory, 1024-aligned:
// two key buffers of PL planes x 128 rows x 128 B, the observation rows (PL x 32 x 128 B), a
// [128][33] fp32 transpose of the logits (pass 0), the MMA barrier, the TMEM address and the
// row statistics (pass 1).
template <int D>
constexpr size_t snap_tile_smem() {
  return (size_t)2 * (D / 64) * kSnapTile * 128 + (size_t)(D / 64) * 32 * 128 + (size_t)kSnapTile * 33 * 4 + 8 +
         16 + 256 + 1024;
}

template <int DT, int D, bool DENSE, int PASS>
__global__ void __launch_bounds__(kSnapTile, 1) snap_tile_kernel(CompressArgs a, int tpc) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int PL = D / 64;  // 128-byte planes of a row
  constexpr uint32_t KBUF = PL * kSnapTile * 128;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  unsigned char* sK = smem;                       // 2 buffers of PL x 128 rows x 128 B
  unsigned char* sQ = smem + 2 * KBUF;            // PL x 32 rows x 128 B
  float* sX = reinterpret_cast<float*>(sQ + PL * 32 * 128);  // [128][33]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sX + kSnapTile * 33);
  uint32_t* sT = reinterpret_cast<uint32_t*>(bar + 1);
  float* sStat = reinterpret_cast<float*>(sT + 4);  // [32][2] row max and sum (pass 1)
  const int h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const hc_layer& L = a.L;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  if (!pl.active) return;
  const int S = pl.S;
  const int tile0 = blockIdx.x * tpc;
  if (tile0 * kSnapTile >= S) return;
  const int ntile = min(tpc, (S - tile0 * kSnapTile + kSnapTile - 1) / kSnapTile);
  const int tqu = min(min(pl.nobs, a.tq), 32);
  if (tqu <= 0) return;
  const int NP = (tqu + 15) & ~15;  // the MMA's N: 16 or 32
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (PASS == 1 && tid < tqu) {
    const float* st = a.stats + (((size_t)s * L.Hk + h) * a.tqmax + tid) * 2;
    sStat[2 * tid] = st[0];
    sStat[2 * tid + 1] = st[1];
  }
  // keys of tile `tile0 + i` into buffer i & 1 (rows past the sequence read as zeros); 16-byte
  // chunk c of row r at plane c/8, chunk (c%8) ^ (r%8): the tensor cores' 128-byte swizzle
  auto load_tile = [&](int i) {
    unsigned char* buf = sK + (i & 1) * KBUF;
    const int t0 = (tile0 + i) * kSnapTile, nt = min(kSnapTile, S - t0);
    for (int k = tid; k < kSnapTile * PL * 8; k += kSnapTile) {
      const int r = k / (PL * 8), c = k % (PL * 8), t = t0 + r;
      const T* src = reinterpret_cast<const T*>(a.q_obs);
      int nb = 0;
      if (r < nt) {
        if constexpr (DENSE) {
          src = reinterpret_cast<const T*>(a.src_k) + (size_t)s * a.ss_seq + (size_t)h * a.ss_head + (size_t)t * a.ss_tok;
          nb = 16;
        } else {
          const int slot = d.hot_ord[t];
          if (slot >= 0 && slot < d.cap) {
            src = reinterpret_cast<const T*>(d.hot_k) + ((size_t)h * d.cap + slot) * D;
            nb = 16;
          } else if ((c & 7) == 0) {
            set_status(d.st, HC_DEV_INDEX);
          }
        }
      }
      cp_async16(buf + (size_t)(c >> 3) * kSnapTile * 128 + (size_t)r * 128 + (((c & 7) ^ (r & 7)) << 4),
                 nb ? src + c * 8 : src, nb);
    }
    cp_async_commit();
  };
  const T* qb = reinterpret_cast<const T*>(a.qb) + ((size_t)s * L.Hk + h) * 32 * D;
  for (int k = tid; k < NP * PL * 8; k += kSnapTile) {
    const int n = k / (PL * 8), c = k % (PL * 8);
    cp_async16(sQ + (size_t)(c >> 3) * NP * 128 + (size_t)n * 128 + (((c & 7) ^ (n & 7)) << 4), qb + (size_t)n * D + c * 8,
               16);
  }
  load_tile(0);  // one group with the observation rows
  if (warp == 0) tmem_alloc(sT, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *sT;
  constexpr uint32_t fmt = DT == HC_BF16 ? 1u : 0u;
  const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(NP >> 3) << 17) |
                         ((uint32_t)(kSnapTile >> 4) << 24);
  for (int i = 0; i < ntile; ++i) {
    if (i + 1 < ntile) {
      load_tile(i + 1);  // lands while tile i is multiplied
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    fence_proxy_async_smem();  // the tensor cores read what cp.async wrote
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t kb = smem_u32(sK) + (uint32_t)(i & 1) * KBUF;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const uint32_t pl2 = ks >> 2, kin = ks & 3;
        const uint32_t aa = kb + pl2 * kSnapTile * 128u + kin * 32u;
        const uint32_t bb = smem_u32(sQ) + pl2 * (uint32_t)NP * 128u + kin * 32u;
        umma_f16(tbase, umma_desc_k_sw128(aa), umma_desc_k_sw128(bb), idesc, ks > 0);
      }
      umma_commit(bar);
    }
    if (!__syncthreads_and(mbar_wait(bar, (uint32_t)(i & 1))) && tid == 0) set_status(d.st, HC_DEV_TIMEOUT);
    tc_fence_after();
    float v[32];
#pragma unroll
    for (int c = 0; c < 32; c += 8)
      if (c < NP) tmem_ld_x8(tbase + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v + c);
    tc_fence_before();
    // logits of token t = t0 + tid; observation row r sits at S - tqu + r and masks later keys
    // (scoring.py:72-74)
    const int t0 = (tile0 + i) * kSnapTile, nt = min(kSnapTile, S - t0), t = t0 + tid;
#pragma unroll
    for (int r = 0; r < 32; ++r)
      v[r] = (r < tqu && tid < nt && t <= S - tqu + r) ? v[r] * L.scale : kNegInf;
    if constexpr (PASS == 0) {
      // per-warp (32-token) partials of every row: the logits go through shared memory so that
      // lane r of warp w reduces row r over the warp's tokens without shuffles
#pragma unroll
      for (int r = 0; r < 32; ++r) sX[tid * 33 + r] = v[r];
      __syncthreads();
      const int chunk = (tile0 + i) * (kSnapTile / 32) + warp;
      if (lane < tqu && chunk * 32 < S) {  // the partials cover ceil(S / 32) chunks
        const float* col = sX + (size_t)warp * 32 * 33 + lane;
        float m = kNegInf;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) m = fmaxf(m, col[j * 33]);
        float l = 0.f;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
          const float x = col[j * 33];
          l += (x == kNegInf) ? 0.f : __expf(x - m);
        }
        float* pp = a.part + ((((size_t)s * L.Hk + h) * a.tqmax + lane) * a.max_chunks + chunk) * 2;
        pp[0] = m;
        pp[1] = l;
      }
    } else {
      if (tid < nt) {
        float acc = 0.f;
        for (int r = 0; r < tqu; ++r) acc += (v[r] == kNegInf) ? 0.f : __expf(v[r] - sStat[2 * r]) / sStat[2 * r + 1];
        a.imp[((size_t)s * L.Hk + h) * a.S_max + t] = acc;
      }
    }
    __syncthreads();  // TMEM and the transpose are free for the next tile
  }
  if (warp == 0) tmem_dealloc(tbase, 32);
}

// ------------------------------------------------------------------------------------------
// SnapKV softmax statistics and token scores
// ------------------------------------------------------------------------------------------
// Per (head, row): max and sum of exp over the whole sequence from the chunk partials. A warp
// per row; grid (ceil(Hk * tqmax / 8), n_seq) of 256 threads.
template <bool DENSE>
__global__ void stats_kernel(CompressArgs a) {
  const hc_layer& L = a.L;
  const int s = blockIdx.y, lane = threadIdx.x & 31;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  if (!pl.active) return;
  const int tqu = min(pl.nobs, a.tq);
  const int nch = (pl.S + a.chunk_len - 1) / a.chunk_len;
  const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (i >= L.Hk * tqu) return;
  const int h = i / tqu, r = i % tqu;
  const float2* p = reinterpret_cast<const float2*>(a.part + (((size_t)s * L.Hk + h) * a.tqmax + r) * a.max_chunks * 2);
  float M = kNegInf;
  for (int c = lane; c < nch; c += 32) M = fmaxf(M, p[c].x);
  M = warp_max(M);
  float S = 0.f;
  for (int c = lane; c < nch; c += 32) {
    const float2 q = p[c];
    S += (q.x == kNegInf) ? 0.f : q.y * __expf(q.x - M);
  }
  S = warp_sum(S);
  if (lane == 0) {
    float* o = a.stats + (((size_t)s * L.Hk + h) * a.tqmax + r) * 2;
    o[0] = M;
    o[1] = S;
  }
}

// importance of token t for head h: sum over rows of softmax probabilities (scoring.py:76-77)
__device__ __forceinline__ float snap_imp(const CompressArgs& a, int s, int h, int tqu, int t) {
  float acc = 0.f;
  for (int r = 0; r < tqu; ++r) {
    const size_t row = ((size_t)s * a.L.Hk + h) * a.tqmax + r;
    const float x = a.logits[row * a.S_max + t];
    const float* st = a.stats + row * 2;
    acc += (x == kNegInf) ? 0.f : __expf(x - st[0]) / st[1];
  }
  return acc;
}

// token score = mean over KV heads of the pooled importance (scoring.py:40-47,78), or the
// hot/cold score sum_h logit_h / sqrt(D) / Hk (cache.py:68-69).
__device__ __forceinline__ float token_score(const CompressArgs& a, int s, int tqu, int S, int t) {
  const hc_layer& L = a.L;
  if (L.policy == HC_POLICY_HOTCOLD) {
    const float inv = 1.f / sqrtf((float)L.D);
    float acc = 0.f;
    for (int h = 0; h < L.Hk; ++h) acc += a.logits[((size_t)s * L.Hk + h) * a.S_max + t] * inv;
    return acc / (float)L.Hk;
  }
  const int pad = L.pool_kernel > 1 ? L.pool_kernel / 2 : 0;
  float tot = 0.f;
  for (int h = 0; h < L.Hk; ++h) {
    const float* imp = a.imp + ((size_t)s * L.Hk + h) * a.S_max;
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
  return tot / (float)L.Hk;
}

// Large inputs: importance for every (head, token), grid (chunks, n_seq).
template <bool DENSE>
__global__ void imp_kernel(CompressArgs a) {
  const hc_layer& L = a.L;
  const int s = blockIdx.y;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  if (!pl.active) return;
  const int tqu = min(pl.nobs, a.tq);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < L.Hk * pl.S; i += gridDim.x * blockDim.x) {
    const int h = i / pl.S, t = i % pl.S;
    a.imp[((size_t)s * L.Hk + h) * a.S_max + t] = snap_imp(a, s, h, tqu, t);
  }
}

template <bool DENSE>
__global__ void token_kernel(CompressArgs a) {
  const hc_layer& L = a.L;
  const int s = blockIdx.y;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  if (!pl.active) return;
  const int tqu = min(pl.nobs, a.tq);
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < pl.S; t += gridDim.x * blockDim.x)
    a.tok[(size_t)s * a.S_max + t] = token_score(a, s, tqu, pl.S, t);
}

// ------------------------------------------------------------------------------------------
// payload copy of one evicted token into the cold ring (+ index vector), one warp
// ------------------------------------------------------------------------------------------
template <int DT, int D, bool DENSE>
__device__ void evict_one(const CompressArgs& a, const hc_seq_desc& d, int s, int src, int dst) {
  using E = Elem<DT>;
  using T = typename E::T;
  const hc_layer& L = a.L;
  const int lane = threadIdx.x & 31;
  constexpr int PER = (D + 31) / 32;
  if (dst < 0 || dst >= d.ccap || src < 0 || src >= (DENSE ? a.S_dense : d.cap)) {
    if (lane == 0) set_status(d.st, HC_DEV_INDEX);
    return;
  }
  float mean[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) mean[i] = 0.f;
  T* __restrict__ ck = reinterpret_cast<T*>(d.cold_kpre) + (size_t)dst * L.Hk * D;
  T* __restrict__ cv = reinterpret_cast<T*>(d.cold_v) + (size_t)dst * L.Hk * D;
  // heads in groups of 8: all loads of a group first, then the stores (no load waits on a store)
  for (int h0 = 0; h0 < L.Hk; h0 += 8) {
    const int nh = min(8, L.Hk - h0);
    T kr[8][PER], vr[8][PER];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nh) break;
      const int h = h0 + j;
      const T* __restrict__ kp;
      const T* __restrict__ vp;
      if constexpr (DENSE) {
        const size_t off = (size_t)s * a.ss_seq + (size_t)h * a.ss_head + (size_t)src * a.ss_tok;
        kp = reinterpret_cast<const T*>(a.src_kpre) + off;
        vp = reinterpret_cast<const T*>(a.src_v) + off;
      } else {
        const size_t off = ((size_t)h * d.cap + src) * D;
        kp = reinterpret_cast<const T*>(d.hot_kpre) + off;
        vp = reinterpret_cast<const T*>(d.hot_v) + off;
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int dd = lane + 32 * i;
        if (dd < D) {
          kr[j][i] = kp[dd];
          vr[j][i] = vp[dd];
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= nh) break;
      const int h = h0 + j;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int dd = lane + 32 * i;
        if (dd < D) {
          ck[(size_t)h * D + dd] = kr[j][i];
          cv[(size_t)h * D + dd] = vr[j][i];
          mean[i] += E::to_f(kr[j][i]);
        }
      }
    }
  }
  if (lane == 0) d.cold_pos[dst] = DENSE ? a.src_pos[(size_t)s * a.S_dense + src] : d.hot_pos[src];
  // index vector (controller.py:178-182): mean over heads, pad/crop to F, L2-normalise
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

// evict_one with 16-byte copies: the payload moves as uint4 chunks (four per lane in flight),
// the pre-RoPE key rows are staged in this warp's `stage` (Hk * D elements) so that the index
// vector is summed over heads in the same order as evict_one.
template <int DT, int D, bool DENSE>
__device__ void evict_one_vec(const CompressArgs& a, const hc_seq_desc& d, int s, int src, int dst,
                              typename Elem<DT>::T* stage) {
  using E = Elem<DT>;
  using T = typename E::T;
  const hc_layer& L = a.L;
  const int lane = threadIdx.x & 31;
  constexpr int PER = (D + 31) / 32;
  constexpr int CPR = D * (int)sizeof(T) / 16;  // 16-byte chunks per head row
  if (dst < 0 || dst >= d.ccap || src < 0 || src >= (DENSE ? a.S_dense : d.cap)) {
    if (lane == 0) set_status(d.st, HC_DEV_INDEX);
    return;
  }
  const int nq = L.Hk * CPR;
  uint4* ck = reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.cold_kpre) + (size_t)dst * L.Hk * D);
  uint4* cv = reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.cold_v) + (size_t)dst * L.Hk * D);
  uint4* st4 = reinterpret_cast<uint4*>(stage);
  for (int q0 = 0; q0 < nq; q0 += 128) {
    uint4 kr[4], vr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = q0 + u * 32 + lane;
      if (q < nq) {
        const int h = q / CPR, c = q % CPR;
        size_t off;
        const T* kb;
        const T* vb;
        if constexpr (DENSE) {
          off = (size_t)s * a.ss_seq + (size_t)h * a.ss_head + (size_t)src * a.ss_tok;
          kb = reinterpret_cast<const T*>(a.src_kpre);
          vb = reinterpret_cast<const T*>(a.src_v);
        } else {
          off = ((size_t)h * d.cap + src) * D;
          kb = reinterpret_cast<const T*>(d.hot_kpre);
          vb = reinterpret_cast<const T*>(d.hot_v);
        }
        kr[u] = reinterpret_cast<const uint4*>(kb + off)[c];
        vr[u] = reinterpret_cast<const uint4*>(vb + off)[c];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int q = q0 + u * 32 + lane;
      if (q < nq) {
        ck[q] = kr[u];
        cv[q] = vr[u];
        st4[q] = kr[u];
      }
    }
  }
  __syncwarp();
  float mean[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) mean[i] = 0.f;
  for (int h = 0; h < L.Hk; ++h)
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i < D) mean[i] += E::to_f(stage[(size_t)h * D + lane + 32 * i]);
  __syncwarp();  // the stage is free for the next token
  if (lane == 0) d.cold_pos[dst] = DENSE ? a.src_pos[(size_t)s * a.S_dense + src] : d.hot_pos[src];
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

// ------------------------------------------------------------------------------------------
// select: top-k of the prefix, compaction, ring plan (one CTA of 1024 threads per sequence)
// ------------------------------------------------------------------------------------------
template <int DT, int D, bool DENSE>
__global__ void __launch_bounds__(1024) select_kernel(CompressArgs a, int small) {
  const hc_layer& L = a.L;
  const int s = blockIdx.x, tid = threadIdx.x;
  __shared__ int sh[kTopkSmemInts];
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  hc_seq_state* st = d.st;
  const Plan pl = make_plan(L, d.budget, min(seq_len<DENSE>(a, d), a.S_max));
  int* hdr = a.hdr + (size_t)s * 16;
  if (DENSE && !pl.active) {
    // a prompt within the budget is stored whole, in order
    const int S = min(pl.S, d.cap);
    for (int t = tid; t < S; t += blockDim.x) a.keep_src[(size_t)s * a.S_max + t] = t;
    for (int i = tid; i < d.cap - S; i += blockDim.x) d.hot_free[i] = d.cap - 1 - i;
    if (tid == 0) {
      if (pl.S > d.cap) set_status(st, HC_DEV_CAPACITY);
      hdr[4] = 1;
      hdr[5] = S;
      hdr[6] = 0;
      st->n_hot = S;
      st->n_free = d.cap - S;
      st->n_evict = 0;
    }
    return;
  }
  if (!pl.active) {
    if (tid == 0) {
      hdr[4] = 0;
      hdr[5] = 0;
      hdr[6] = 0;
      st->n_evict = 0;
    }
    return;
  }
  const int S = pl.S, tqu = min(pl.nobs, a.tq);
  float* tok = a.tok + (size_t)s * a.S_max;
  uint8_t* sel = a.sel + (size_t)s * a.S_max;

  if (small) {
    // everything in shared memory: logits [rows][S] -> (SnapKV) importance [Hk][S] -> scores [S]
    extern __shared__ __align__(16) float dyn[];
    const bool snap = L.policy == HC_POLICY_SNAPKV;
    const int rows = L.Hk * (snap ? tqu : 1);
    float* sLg = dyn;                      // rows * S
    float* sImp = sLg + (size_t)rows * S;  // Hk * S (SnapKV)
    float* sStat = sImp + (snap ? (size_t)L.Hk * S : 0);  // rows * 2
    float* sTok = sStat + 2 * rows;        // S
    uint8_t* sSel = reinterpret_cast<uint8_t*>(sTok + S);
    for (int row = 0; row < rows; ++row) {  // row by row: no division per element
      const size_t g = snap ? (((size_t)s * L.Hk + row / tqu) * a.tqmax + row % tqu) : ((size_t)s * L.Hk + row);
      const float* src = a.logits + g * a.S_max;
      for (int t = tid; t < S; t += blockDim.x) sLg[(size_t)row * S + t] = src[t];
    }
    __syncthreads();
    if (snap && tqu == 1) {
      // one observation row (decode): each head's softmax statistics from the score kernel's
      // chunk partials, and the max-pooled probability of a window as exp(max logit - M) / L
      // (exp and the division are monotone, so this is the pool of the probabilities)
      const int warp = tid >> 5, lane = tid & 31;
      const int nch = (S + a.chunk_len - 1) / a.chunk_len;
      for (int hh = warp; hh < L.Hk; hh += blockDim.x >> 5) {
        const float* pp = a.part + ((size_t)s * L.Hk + hh) * a.tqmax * a.max_chunks * 2;
        float M = kNegInf;
        for (int c2 = lane; c2 < nch; c2 += 32) M = fmaxf(M, pp[2 * c2]);
        M = warp_max(M);
        float Ls = 0.f;
        for (int c2 = lane; c2 < nch; c2 += 32) Ls += (pp[2 * c2] == kNegInf) ? 0.f : pp[2 * c2 + 1] * __expf(pp[2 * c2] - M);
        Ls = warp_sum(Ls);
        if (lane == 0) {
          sStat[2 * hh] = M;
          sStat[2 * hh + 1] = Ls;
        }
      }
      __syncthreads();
      const int pad = L.pool_kernel > 1 ? L.pool_kernel / 2 : 0;
      const bool pmax = L.pooling == HC_POOL_MAX;
      for (int t = tid; t < S; t += blockDim.x) {
        float tot = 0.f;
        for (int hh = 0; hh < L.Hk; ++hh) {
          const float* lg = sLg + (size_t)hh * S;
          const float M = sStat[2 * hh], Ls = sStat[2 * hh + 1];
          float v;
          if (pad == 0 || pmax) {
            float mx = kNegInf;
            for (int u = max(0, t - pad); u <= min(S - 1, t + pad); ++u) mx = fmaxf(mx, lg[u]);
            v = (mx == kNegInf) ? 0.f : __expf(mx - M) / Ls;
          } else {
            v = 0.f;
            for (int u = max(0, t - pad); u <= min(S - 1, t + pad); ++u)
              v += (lg[u] == kNegInf) ? 0.f : __expf(lg[u] - M) / Ls;
            v /= (float)L.pool_kernel;
          }
          tot += v;
        }
        sTok[t] = tot / (float)L.Hk;
      }
    } else if (snap) {
      const int warp = tid >> 5, lane = tid & 31;
      for (int r = warp; r < rows; r += blockDim.x >> 5) {
        const float* lg = sLg + (size_t)r * S;
        float m = kNegInf;
        for (int t = lane; t < S; t += 32) m = fmaxf(m, lg[t]);
        m = warp_max(m);
        float l = 0.f;
        for (int t = lane; t < S; t += 32) l += (lg[t] == kNegInf) ? 0.f : __expf(lg[t] - m);
        l = warp_sum(l);
        if (lane == 0) {
          sStat[2 * r] = m;
          sStat[2 * r + 1] = l;
        }
      }
      __syncthreads();
      for (int h = 0; h < L.Hk; ++h)
        for (int t = tid; t < S; t += blockDim.x) {
          float acc = 0.f;
          for (int r = 0; r < tqu; ++r) {
            const int row = h * tqu + r;
            const float x = sLg[(size_t)row * S + t];
            acc += (x == kNegInf) ? 0.f : __expf(x - sStat[2 * row]) / sStat[2 * row + 1];
          }
          sImp[(size_t)h * S + t] = acc;
        }
      __syncthreads();
      const int pad = L.pool_kernel > 1 ? L.pool_kernel / 2 : 0;
      for (int t = tid; t < S; t += blockDim.x) {
        float tot = 0.f;
        for (int h = 0; h < L.Hk; ++h) {
          const float* imp = sImp + (size_t)h * S;
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
      for (int t = tid; t < S; t += blockDim.x) {
        float acc = 0.f;
        for (int h = 0; h < L.Hk; ++h) acc += sLg[(size_t)h * S + t] * inv;
        sTok[t] = acc / (float)L.Hk;
      }
    }
    __syncthreads();
    tok = sTok;
    sel = sSel;
  }

  // one eviction from the slab (the decode steady state): the lowest-scoring prefix token,
  // the higher index among equal scores (the top-k keeps the lower one), then the order table
  // shifts down by one past it. Same result as the top-k + compaction below.
  if (!DENSE && pl.prefix - pl.ntop == 1 && S <= 8 * (int)blockDim.x) {
    __shared__ unsigned long long s_min[32];
    unsigned long long m = ~0ull;
    for (int t = tid; t < pl.prefix; t += blockDim.x) {
      const unsigned long long k = ((unsigned long long)fkey(tok[t]) << 32) | (0xffffffffu - (uint32_t)t);
      m = k < m ? k : m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, m, o);
      m = y < m ? y : m;
    }
    if ((tid & 31) == 0) s_min[tid >> 5] = m;
    __syncthreads();
    if (tid < 32) {
      unsigned long long x = tid < (int)(blockDim.x >> 5) ? s_min[tid] : ~0ull;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, x, o);
        x = y < x ? y : x;
      }
      if (tid == 0) s_min[0] = x;
    }
    __syncthreads();
    const int e = (int)(0xffffffffu - (uint32_t)(s_min[0] & 0xffffffffu));
    const int phys_e = d.hot_ord[e];
    int vals[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = e + tid + j * (int)blockDim.x;
      if (t < S - 1) vals[j] = d.hot_ord[t + 1];
    }
    __syncthreads();  // every read of the order table is done
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = e + tid + j * (int)blockDim.x;
      if (t < S - 1) d.hot_ord[t] = vals[j];
    }
    const int ccap = d.ccap, cold_head = st->cold_head, cold_count = st->cold_count, n_free0 = st->n_free;
    const int dst = (int)(((long)cold_head + cold_count) % ccap);
    __syncthreads();  // every thread has read the counters before thread 0 updates them
    if (tid == 0) {
      a.ev_src[(size_t)s * a.S_max] = phys_e;
      a.ev_dst[(size_t)s * a.S_max] = dst;
      if (n_free0 < d.cap) d.hot_free[n_free0] = phys_e;
      const long total = (long)cold_count + 1;
      if (total > ccap) {
        st->cold_head = (int)(((long)cold_head + total - ccap) % ccap);
        st->cold_count = ccap;
      } else {
        st->cold_count = (int)total;
      }
      st->n_evict = 1;
      st->n_hot = S - 1;
      st->n_free = n_free0 + 1;
      hdr[0] = S;
      hdr[4] = 1;
      hdr[5] = 0;
      hdr[6] = 1;
    }
    if (tid < 32) evict_one<DT, D, false>(a, d, s, phys_e, dst);
    return;
  }

  // exact top-n_top of the prefix. Up to kRangeMax tokens per thread, each thread takes a
  // contiguous range (a few block-wide steps in all); longer prompts keep the coalesced passes
  // over blockDim-token chunks (per-thread loops over long ranges serialise their loads)
  constexpr int kRangeMax = 8;
  const int per = (S + (int)blockDim.x - 1) / (int)blockDim.x;
  if (per <= kRangeMax) block_topk_ranges([&](int i) { return tok[i]; }, pl.prefix, pl.ntop, sel, sh);
  else block_topk_flags([&](int i) { return tok[i]; }, pl.prefix, pl.ntop, sel, sh);

  // order-preserving compaction. keep: selected prefix tokens and the tail; evict: the rest
  int kept = 0, evicted = 0;
  const int n_evict_total = pl.prefix - pl.ntop;
  const int ccap = d.ccap;
  const int cold_head = st->cold_head, cold_count = st->cold_count;
  const int n_free0 = DENSE ? 0 : st->n_free;
  if (per <= kRangeMax) {
    // thread t owns tokens [t * per, (t + 1) * per): counts, one block scan of (kept | evicted
    // << 16) when both fit 16 bits (else two scans), then the thread writes its run in order
    // (the slab's order table is read into registers first)
    const int r0 = min(S, tid * per), r1 = min(S, r0 + per);
    int nk = 0, ne = 0;
    int phys[kRangeMax];
    for (int i = r0; i < r1; ++i) {
      const bool keep = (i >= pl.prefix) || sel[i];
      nk += keep;
      ne += !keep;
      if (!DENSE) phys[i - r0] = d.hot_ord[i];
    }
    int kb, eb, tk, te;
    if (S < 65536) {
      int tot;
      const int b = block_exclusive_scan(nk | (ne << 16), sh + 256, tot);
      kb = b & 0xffff;
      eb = b >> 16;
      tk = tot & 0xffff;
      te = tot >> 16;
    } else {
      kb = block_exclusive_scan(nk, sh + 256, tk);
      eb = block_exclusive_scan(ne, sh + 256, te);
    }
    // the scans end with a barrier: every order-table read above is done before the writes
    for (int i = r0; i < r1; ++i) {
      const bool keep = (i >= pl.prefix) || sel[i];
      const int ph = DENSE ? -1 : phys[i - r0];
      if (keep) {
        if (DENSE) a.keep_src[(size_t)s * a.S_max + kb] = i;
        else d.hot_ord[kb] = ph;
        ++kb;
      } else {
        const int j = eb++;
        a.ev_src[(size_t)s * a.S_max + j] = DENSE ? i : ph;
        // ring slot of the j-th evicted token; a batch larger than the ring keeps its last ccap
        a.ev_dst[(size_t)s * a.S_max + j] =
            (j >= n_evict_total - ccap) ? (int)(((long)cold_head + cold_count + j) % ccap) : -1;
        if (!DENSE && n_free0 + j < d.cap) d.hot_free[n_free0 + j] = ph;
      }
    }
    kept = tk;
    evicted = te;
    __syncthreads();
  } else
  for (int base = 0; base < S; base += blockDim.x) {
    const int t = base + tid;
    int keep = 0, ev = 0, phys = -1;
    if (t < S) {
      keep = (t >= pl.prefix) || sel[t];
      ev = !keep;
      if (!DENSE) phys = d.hot_ord[t];
    }
    int tk, te;
    const int rk = block_exclusive_scan(keep, sh + 256, tk);
    const int re = block_exclusive_scan(ev, sh + 256, te);
    // block_exclusive_scan ends with a barrier, so every hot_ord read above is done
    if (t < S) {
      if (keep) {
        if (DENSE) a.keep_src[(size_t)s * a.S_max + kept + rk] = t;
        else d.hot_ord[kept + rk] = phys;
      } else {
        const int j = evicted + re;
        const int src = DENSE ? t : phys;
        a.ev_src[(size_t)s * a.S_max + j] = src;
        // ring slot of the j-th evicted token; a batch larger than the ring keeps its last ccap
        a.ev_dst[(size_t)s * a.S_max + j] =
            (j >= n_evict_total - ccap) ? (int)(((long)cold_head + cold_count + j) % ccap) : -1;
        if (!DENSE && n_free0 + j < d.cap) d.hot_free[n_free0 + j] = phys;
      }
    }
    kept += tk;
    evicted += te;
    __syncthreads();
  }
  if (tid == 0) {
    const long total = (long)cold_count + evicted;
    int nh = cold_head, nc = (int)total;
    if (total > ccap) {
      nh = (int)(((long)cold_head + total - ccap) % ccap);
      nc = ccap;
    }
    st->cold_head = nh;
    st->cold_count = nc;
    st->n_evict = evicted;
    if (DENSE) {
      st->n_hot = kept;
      st->n_free = d.cap - kept;
    } else {
      st->n_hot = kept;
      st->n_free = n_free0 + evicted;
    }
    hdr[0] = S;
    hdr[4] = 1;
    hdr[5] = DENSE ? kept : 0;
    hdr[6] = evicted;
  }
  if (DENSE) {
    for (int i = tid; i < d.cap - kept; i += blockDim.x) d.hot_free[i] = d.cap - 1 - i;
  }
  // small decode evictions: copy here, one warp per token
  if (!DENSE && evicted <= kInlineEvict) {
    __syncthreads();
    const int warp = tid >> 5;
    for (int j = warp; j < evicted; j += 32) {
      const int dst = a.ev_dst[(size_t)s * a.S_max + j];
      if (dst >= 0) evict_one<DT, D, false>(a, d, s, a.ev_src[(size_t)s * a.S_max + j], dst);
    }
  }
}

// ------------------------------------------------------------------------------------------
// select for a prompt: the same keep / evict lists as select_kernel, from a cluster of C CTAs
// per sequence (grid (C, n_seq), cluster (C, 1, 1), 1024 threads; C * 1024 * kSelPer >= S)
// ------------------------------------------------------------------------------------------
constexpr int kSelPer = 8;     // most tokens per thread of the prompt selection (keys in registers)
constexpr int kSelTarget = 2;  // tokens per thread the cluster is sized for, up to 16 CTAs

// Warp 0 finds the radix digit holding the kk-th largest key of a 256-bin histogram (bins in
// ascending key order): misc[0] = digit, misc[1] = rank of the k-th largest inside the bin.
__device__ __forceinline__ void radix_digit(const int* hist, int kk, int* misc) {
  const int lane = threadIdx.x & 31;
  int tot = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) tot += hist[255 - 8 * lane - j];
  int inc = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  const int excl = inc - tot;
  const unsigned hit = __ballot_sync(0xffffffffu, inc >= kk && excl < kk);
  if (lane == __ffs(hit) - 1) {
    int cum = excl, digit = 0;
    for (int j = 0; j < 8; ++j) {
      const int b = 255 - 8 * lane - j;
      if (cum + hist[b] >= kk) {
        digit = b;
        break;
      }
      cum += hist[b];
    }
    misc[0] = digit;
    misc[1] = kk - cum;
  }
}

// Thread g = rank * 1024 + tid owns tokens [g * per, (g + 1) * per), per = ceil(S / (C * 1024)).
// The top-n_top of the prefix is an exact MSB radix select over the order-preserving keys
// (four 8-bit passes): each CTA builds its histogram with warp-aggregated shared atomics, and
// after one cluster barrier every CTA sums the C histograms through distributed shared memory
// and finds the same digit (histograms double-buffered, so a pass needs one cluster barrier).
// The threshold key T and the number kk of tokens equal to T that are kept then fix every
// position: with gt(p) / eq(p) the prefix tokens before p above / equal to T, the kept tokens
// before p number gt(p) + min(kk, eq(p)) + (tail tokens before p) — ties go to the lower index
// as in block_topk_flags — and the evicted ones min(p, prefix) - gt(p) - min(kk, eq(p)). One
// block scan of (gt | eq << 16) per thread and one exchange of the CTA totals give them.
// With `fused`, the token scores (token_score: pooled importance averaged over KV heads) are
// computed here, CTA c scoring its own tokens [c * 1024 * per, (c + 1) * 1024 * per) with
// coalesced loads into shared memory, from which each thread takes its range; otherwise they
// come from token_kernel.
__global__ void __launch_bounds__(1024) select_cluster_kernel(CompressArgs a, int fused) {
  const hc_layer& L = a.L;
  const int s = blockIdx.y, tid = threadIdx.x, C = gridDim.x, rank = blockIdx.x;
  __shared__ int hist[2][256];
  __shared__ int tot[256];
  __shared__ int misc[2];
  __shared__ int scan_sh[40];
  __shared__ int pub;       // this CTA's packed (gt | eq << 16) count, read by the cluster
  __shared__ int ctot[16];  // the C CTAs' packed counts
  __shared__ float sTok[1024 * kSelPer];
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  hc_seq_state* st = d.st;
  const Plan pl = make_plan(L, d.budget, min(a.S_dense, a.S_max));
  int* hdr = a.hdr + (size_t)s * 16;
  const int g = rank * (int)blockDim.x + tid, nthr = C * (int)blockDim.x;
  if (!pl.active) {
    // a prompt within the budget is stored whole, in order (every CTA of the cluster returns
    // here, before any cluster barrier)
    const int S = min(pl.S, d.cap);
    for (int t = g; t < S; t += nthr) a.keep_src[(size_t)s * a.S_max + t] = t;
    for (int i = g; i < d.cap - S; i += nthr) d.hot_free[i] = d.cap - 1 - i;
    if (g == 0) {
      if (pl.S > d.cap) set_status(st, HC_DEV_CAPACITY);
      hdr[4] = 1;
      hdr[5] = S;
      hdr[6] = 0;
      st->n_hot = S;
      st->n_free = d.cap - S;
      st->n_evict = 0;
    }
    return;
  }
  const int S = pl.S, P = pl.prefix, K = pl.ntop;
  const int per = (S + nthr - 1) / nthr;
  const int r0 = min(S, g * per), r1 = min(S, r0 + per), npre = max(0, min(r1, P) - r0);
  // ring state, read by every thread before the CTA of rank 0 updates it (after the count
  // exchange's cluster barrier)
  const int ccap = d.ccap, cold_head = st->cold_head, cold_count = st->cold_count;
  uint32_t key[kSelPer];
  if (fused) {
    const int tqu = min(pl.nobs, a.tq);
    const int c0 = min(S, rank * (int)blockDim.x * per), c1 = min(S, c0 + (int)blockDim.x * per);
    for (int i = c0 + tid; i < c1; i += blockDim.x) sTok[i - c0] = token_score(a, s, tqu, S, i);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kSelPer; ++j) key[j] = j < npre ? fkey(sTok[tid * per + j]) : 0u;
  } else {
    const float* tok = a.tok + (size_t)s * a.S_max;
#pragma unroll
    for (int j = 0; j < kSelPer; ++j) key[j] = j < npre ? fkey(tok[r0 + j]) : 0u;
  }
  const bool all = K >= P, none = K <= 0;
  uint32_t T = 0;
  int kk = 0;
  if (!all && !none) {
    uint32_t pre = 0, mask = 0;
    kk = K;
    if (tid < 256) hist[0][tid] = 0;
    __syncthreads();
#pragma unroll 1
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      int* hb = hist[pass & 1];
#pragma unroll
      for (int j = 0; j < kSelPer; ++j) {
        const bool live = j < npre && (key[j] & mask) == pre;
        const unsigned act = __ballot_sync(0xffffffffu, live);
        if (live) {
          const uint32_t bin = (key[j] >> shift) & 255u;
          const unsigned same = __match_any_sync(act, bin);
          if ((tid & 31) == __ffs(same) - 1) atomicAdd(&hb[bin], __popc(same));
        }
      }
      __syncthreads();
      cluster_arrive();
      cluster_wait();
      // the other buffer was last read by the cluster in the previous pass, before every CTA
      // arrived at the barrier just passed
      if (tid < 256) {
        hist[(pass + 1) & 1][tid] = 0;
        int acc = 0;
        for (int r = 0; r < C; ++r) acc += ld_cluster_s32(&hb[tid], (uint32_t)r);
        tot[tid] = acc;
      }
      __syncthreads();
      if (tid < 32) radix_digit(tot, kk, misc);
      __syncthreads();
      pre |= (uint32_t)misc[0] << shift;
      mask |= 255u << shift;
      kk = misc[1];
    }
    T = pre;
  }
  int ngt = 0, neq = 0;
#pragma unroll
  for (int j = 0; j < kSelPer; ++j) {
    if (j < npre) {
      ngt += all || (!none && key[j] > T);
      neq += !all && !none && key[j] == T;
    }
  }
  int ctotal;
  const int before = block_exclusive_scan(ngt | (neq << 16), scan_sh, ctotal);
  if (tid == 0) pub = ctotal;
  cluster_arrive();
  cluster_wait();
  if (tid < C) ctot[tid] = ld_cluster_s32(&pub, (uint32_t)tid);
  __syncthreads();
  // every read of the cluster's shared memory is done: arrive now, wait before exiting
  cluster_arrive_relaxed();
  int gt_p = before & 0xffff, eq_p = before >> 16, gt_all = 0, eq_all = 0;
  for (int r = 0; r < C; ++r) {
    const int v = ctot[r];
    if (r < rank) {
      gt_p += v & 0xffff;
      eq_p += v >> 16;
    }
    gt_all += v & 0xffff;
    eq_all += v >> 16;
  }
  const int taken_all = gt_all + min(kk, eq_all);
  const int n_evict_total = P - taken_all, kept = S - n_evict_total;
  int kb = gt_p + min(kk, eq_p) + max(0, r0 - P);
  int eb = min(r0, P) - gt_p - min(kk, eq_p);
  int eqr = eq_p;
#pragma unroll
  for (int j = 0; j < kSelPer; ++j) {
    const int i = r0 + j;
    if (i < r1) {
      bool keep = true;
      if (j < npre) {
        keep = all || (!none && key[j] > T);
        if (!all && !none && key[j] == T) keep = eqr++ < kk;
      }
      if (keep) {
        a.keep_src[(size_t)s * a.S_max + kb++] = i;
      } else {
        const int e = eb++;
        a.ev_src[(size_t)s * a.S_max + e] = i;
        // ring slot of the e-th evicted token; a batch larger than the ring keeps its last ccap
        a.ev_dst[(size_t)s * a.S_max + e] =
            (e >= n_evict_total - ccap) ? (int)(((long)cold_head + cold_count + e) % ccap) : -1;
      }
    }
  }
  for (int i = g; i < d.cap - kept; i += nthr) d.hot_free[i] = d.cap - 1 - i;
  if (g == 0) {
    const long total = (long)cold_count + n_evict_total;
    int nh = cold_head, nc = (int)total;
    if (total > ccap) {
      nh = (int)(((long)cold_head + total - ccap) % ccap);
      nc = ccap;
    }
    st->cold_head = nh;
    st->cold_count = nc;
    st->n_evict = n_evict_total;
    st->n_hot = kept;
    st->n_free = d.cap - kept;
    hdr[0] = S;
    hdr[4] = 1;
    hdr[5] = kept;
    hdr[6] = n_evict_total;
  }
  cluster_wait();
}

// Large evictions and the prompt store: kept tokens -> slab slots 0..n_keep-1 (prompt),
// evicted tokens -> cold ring. Grid (blocks, n_seq), 8 warps per block, a warp per token.
template <int DT, int D, bool DENSE>
__global__ void __launch_bounds__(256) evict_kernel(CompressArgs a) {
  using T = typename Elem<DT>::T;
  const hc_layer& L = a.L;
  const int s = blockIdx.y;
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  const int* hdr = a.hdr + (size_t)s * 16;
  if (!hdr[4]) return;
  const int n_keep = hdr[5], n_ev = hdr[6];
  if (!DENSE && n_ev <= kInlineEvict) return;
  const int lane = threadIdx.x & 31;
  const int w0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, nw = (gridDim.x * blockDim.x) >> 5;
  if (a.vec_ok) {
    extern __shared__ __align__(16) unsigned char evs[];
    T* stage = reinterpret_cast<T*>(evs) + (size_t)(threadIdx.x >> 5) * L.Hk * D;
    constexpr int CPR = D * (int)sizeof(T) / 16;
    for (int item = w0; item < n_keep + n_ev; item += nw) {
      if (item < n_keep) {
        if constexpr (DENSE) {
          const int t = a.keep_src[(size_t)s * a.S_max + item];
          for (int q = lane; q < L.Hk * CPR; q += 32) {
            const int h = q / CPR, c = q % CPR;
            const size_t src = (size_t)s * a.ss_seq + (size_t)h * a.ss_head + (size_t)t * a.ss_tok;
            const size_t dst = ((size_t)h * d.cap + item) * D;
            const uint4 kx = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.src_k) + src)[c];
            const uint4 vx = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.src_v) + src)[c];
            const uint4 px = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.src_kpre) + src)[c];
            reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.hot_k) + dst)[c] = kx;
            reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.hot_v) + dst)[c] = vx;
            reinterpret_cast<uint4*>(reinterpret_cast<T*>(d.hot_kpre) + dst)[c] = px;
          }
          if (lane == 0) {
            d.hot_pos[item] = a.src_pos[(size_t)s * a.S_dense + t];
            d.hot_ord[item] = item;
          }
        }
      } else {
        const int j = item - n_keep;
        const int dst = a.ev_dst[(size_t)s * a.S_max + j];
        if (dst >= 0) evict_one_vec<DT, D, DENSE>(a, d, s, a.ev_src[(size_t)s * a.S_max + j], dst, stage);
      }
    }
    return;
  }
  for (int item = w0; item < n_keep + n_ev; item += nw) {
    if (item < n_keep) {
      if constexpr (DENSE) {
        const int t = a.keep_src[(size_t)s * a.S_max + item];
        for (int h = 0; h < L.Hk; ++h) {
          const size_t src = (size_t)s * a.ss_seq + (size_t)h * a.ss_head + (size_t)t * a.ss_tok;
          const size_t dst = ((size_t)h * d.cap + item) * D;
          for (int dd = lane; dd < D; dd += 32) {
            reinterpret_cast<T*>(d.hot_k)[dst + dd] = reinterpret_cast<const T*>(a.src_k)[src + dd];
            reinterpret_cast<T*>(d.hot_v)[dst + dd] = reinterpret_cast<const T*>(a.src_v)[src + dd];
            reinterpret_cast<T*>(d.hot_kpre)[dst + dd] = reinterpret_cast<const T*>(a.src_kpre)[src + dd];
          }
        }
        if (lane == 0) {
          d.hot_pos[item] = a.src_pos[(size_t)s * a.S_dense + t];
          d.hot_ord[item] = item;
        }
      }
    } else {
      const int j = item - n_keep;
      const int dst = a.ev_dst[(size_t)s * a.S_max + j];
      if (dst >= 0) evict_one<DT, D, DENSE>(a, d, s, a.ev_src[(size_t)s * a.S_max + j], dst);
    }
  }
}

// Stand-alone cold append (add_evicted_to_cold_store, controller.py:190-238): tokens with
// evicted_idx >= 0 in index order; a batch larger than the ring keeps its newest ccap.
// One CTA of 256 threads per sequence.
template <int DT, int D>
__global__ void __launch_bounds__(256) cold_append_kernel(CompressArgs a, const int64_t* idx, int Te) {
  const hc_layer& L = a.L;
  const int s = blockIdx.x, tid = threadIdx.x;
  __shared__ int sh[64];
  __shared__ int sdst[1024];
  __shared__ int ssrc[1024];
  pdl_wait();
  const hc_seq_desc d = L.desc[s];
  hc_seq_state* st = d.st;
  const int head = st->cold_head, count = st->cold_count, ccap = d.ccap;
  // number of valid tokens
  int m = 0;
  for (int base = 0; base < Te; base += blockDim.x) {
    const int t = base + tid;
    int tot;
    block_exclusive_scan((t < Te && idx[(size_t)s * Te + t] >= 0) ? 1 : 0, sh, tot);
    m += tot;
  }
  int j0 = 0;
  for (int base = 0; base < Te; base += blockDim.x) {
    const int t = base + tid;
    const int f = (t < Te && idx[(size_t)s * Te + t] >= 0) ? 1 : 0;
    int tot;
    const int r = block_exclusive_scan(f, sh, tot);
    if (f) {
      const int j = j0 + r;
      ssrc[tid] = t;
      sdst[tid] = (j >= m - ccap) ? (int)(((long)head + count + j) % ccap) : -1;
    } else {
      sdst[tid] = -2;
    }
    __syncthreads();
    for (int w = tid >> 5; w < (int)blockDim.x; w += blockDim.x >> 5) {
      const int dst = sdst[w];
      if (dst >= 0) evict_one<DT, D, true>(a, d, s, ssrc[w], dst);
    }
    __syncthreads();
    j0 += tot;
  }
  if (tid == 0) {
    const long total = (long)count + m;
    if (total > ccap) {
      st->cold_head = (int)(((long)head + total - ccap) % ccap);
      st->cold_count = ccap;
    } else {
      st->cold_count = (int)total;
    }
  }
}

template <int DT, int D>
static cudaError_t cold_append_t(CompressArgs a, const int64_t* idx, int Te, cudaStream_t stream) {
  return launch_pdl(cold_append_kernel<DT, D>, dim3(a.L.n_seq), dim3(256), 0, stream, a, idx, Te);
}

cudaError_t launch_cold_append(const hc_layer& L, const void* kpre, const void* v, int64_t s0, int64_t s1, int64_t s2,
                               const int64_t* pos, const int64_t* idx, int Te, cudaStream_t stream) {
  CompressArgs a{};
  a.L = L;
  a.src_kpre = kpre;
  a.src_v = v;
  a.ss_seq = s0; a.ss_head = s1; a.ss_tok = s2;
  a.src_pos = pos;
  a.S_dense = Te;
  HC_DISPATCH_DT_D(L.dtype, L.D, cold_append_t, a, idx, Te, stream);
}

// ------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------
struct CompressLayout {
  size_t hdr, logits, part, stats, imp, tok, sel, keep_src, ev_src, ev_dst, qb, total;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

CompressLayout compress_layout(const hc_layer& L, int S_max, int tq) {
  CompressLayout c{};
  const size_t n = (size_t)L.n_seq, Hk = (size_t)L.Hk, S = (size_t)S_max;
  const size_t tqm = (size_t)(tq > 0 ? tq : 1);
  const size_t chunks = (S + 31) / 32;  // softmax partials of 32 (tensor-core path) or 64 tokens
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align256(bytes); return o; };
  c.hdr = take(n * 16 * sizeof(int));
  c.logits = take(n * Hk * tqm * S * sizeof(float));
  c.part = take(n * Hk * tqm * chunks * 2 * sizeof(float));
  c.stats = take(n * Hk * tqm * 2 * sizeof(float));
  c.imp = take(n * Hk * S * sizeof(float));
  c.tok = take(n * S * sizeof(float));
  c.sel = take(n * S);
  c.keep_src = take(n * S * sizeof(int));
  c.ev_src = take(n * S * sizeof(int));
  c.ev_dst = take(n * S * sizeof(int));
  c.qb = take(n * Hk * 32 * (size_t)L.D * 2);
  c.total = off;
  return c;
}

// Launch configuration of the prompt selection: a cluster of C CTAs per sequence.
static cudaLaunchConfig_t select_cluster_config(cudaLaunchAttribute* attr, int C, int n_seq, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, n_seq);
  cfg.blockDim = dim3(1024);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cfg;
}

// Whether the device holds a cluster of C CTAs of the prompt selection (clusters above 8 CTAs
// are non-portable; checked once per device).
static cudaError_t select_cluster_fits(int C, bool& fits) {
  fits = true;
  if (C <= 8) return cudaSuccess;
  static std::mutex mu;
  static int ok_dev[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  const int di = dev & 63;
  if (ok_dev[di] == 0) {
    e = cudaFuncSetAttribute(select_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg = select_cluster_config(attr, C, 1, nullptr);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, select_cluster_kernel, &cfg);
    if (e != cudaSuccess) return e;
    ok_dev[di] = clusters >= 1 ? 1 : -1;
  }
  fits = ok_dev[di] > 0;
  return cudaSuccess;
}

template <int DT, int D, bool DENSE>
static cudaError_t compress_t(CompressArgs a, int S_grid, int n_evict_hint, cudaStream_t stream) {
  using T = typename Elem<DT>::T;
  const hc_layer& L = a.L;
  // the selection CTA computes the token scores itself when its inputs fit shared memory
  const bool snap = L.policy == HC_POLICY_SNAPKV;
  const size_t rows = (size_t)L.Hk * (snap ? a.tqmax : 1);
  const size_t sel_smem =
      4 * (rows * S_grid + (snap ? (size_t)L.Hk * S_grid : 0) + 2 * rows + (size_t)S_grid) + S_grid + 64;
  const int small = sel_smem <= kSelectSmemMax ? 1 : 0;
  // large SnapKV inputs of 16-bit layers: the observation x prefix product on the tensor cores
  const bool tc = snap && !small && DT != HC_F32 && (D % 64) == 0 && min(L.recent, a.tq) <= 32;
  cudaError_t e = cudaSuccess;
  if (tc) {
    a.chunk_len = 32;
    const int tiles = (S_grid + kSnapTile - 1) / kSnapTile;
    // tiles per CTA: about two CTAs per SM over the whole grid
    const long all_tiles = (long)tiles * L.Hk * L.n_seq;
    int tpc = (int)((all_tiles + 295) / 296);
    tpc = tpc < 1 ? 1 : tpc > 16 ? 16 : tpc;
    const int gx = (tiles + tpc - 1) / tpc;
    const size_t tsmem = snap_tile_smem<D>();
    auto k0 = snap_tile_kernel<DT, D, DENSE, 0>;
    auto k1 = snap_tile_kernel<DT, D, DENSE, 1>;
    e = ensure_smem(k0, tsmem);
    if (e == cudaSuccess) e = ensure_smem(k1, tsmem);
    if (e != cudaSuccess) return e;
    e = launch_pdl(snap_qbar_kernel<DT, D, DENSE>, dim3(L.Hk, 16, L.n_seq), dim3(256), 0, stream, a);
    if (e == cudaSuccess) e = launch_pdl(k0, dim3(gx, L.Hk, L.n_seq), dim3(kSnapTile), tsmem, stream, a, tpc);
    if (e == cudaSuccess)
      e = launch_pdl(stats_kernel<DENSE>, dim3((L.Hk * a.tqmax + 7) / 8, L.n_seq), dim3(256), 0, stream, a);
    if (e == cudaSuccess) e = launch_pdl(k1, dim3(gx, L.Hk, L.n_seq), dim3(kSnapTile), tsmem, stream, a, tpc);
    if (e != cudaSuccess) return e;
  } else {
    const size_t smem = sizeof(T) * kScoreCH * D +
                        sizeof(float) * ((size_t)(a.tqmax + 1) * D + (size_t)a.tqmax * kScoreCH) + 64 +
                        sizeof(void*) * kScoreCH;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    auto sk = score_kernel<DT, D, DENSE>;
    e = ensure_smem(sk, 200 * 1024);
    if (e != cudaSuccess) return e;
    const int chunks = (S_grid + kScoreCH - 1) / kScoreCH;
    e = launch_pdl(sk, dim3(chunks, L.Hk, L.n_seq), dim3(128), smem, stream, a);
    if (e != cudaSuccess) return e;
  }
  // A long prompt's selection runs on a cluster: up to 16k tokens one token per thread, the
  // token scores computed by the cluster itself (their pooled loads are bound by each SM's L2
  // bandwidth, so they gain only when spread that thin); longer prompts on up to 16 CTAs sized
  // for kSelTarget tokens per thread, after token_kernel. Short prompts (scored in shared
  // memory) and decode steps select on one CTA.
  int C = 0, fused = 0;
  if (DENSE && !small) {
    C = 1;
    if (S_grid <= 16 * 1024) {
      while (C * 1024 < S_grid) C <<= 1;
      fused = 1;
    } else {
      while (C < 16 && (long)C * 1024 * kSelTarget < S_grid) C <<= 1;
    }
    if (C > 8) {
      bool fits = true;
      e = select_cluster_fits(C, fits);
      if (e != cudaSuccess) return e;
      if (!fits) {
        C = 8;
        fused = 0;
      }
    }
    if ((long)C * 1024 * kSelPer < S_grid) C = fused = 0;
  }
  if (!small) {
    const int blocks = (int)((S_grid + 255) / 256) < 592 ? (S_grid + 255) / 256 : 592;
    if (snap && !tc) {
      e = launch_pdl(stats_kernel<DENSE>, dim3((L.Hk * a.tqmax + 7) / 8, L.n_seq), dim3(256), 0, stream, a);
      if (e != cudaSuccess) return e;
      const int ib = (int)(((long)L.Hk * S_grid + 255) / 256) < 1184 ? (int)(((long)L.Hk * S_grid + 255) / 256) : 1184;
      e = launch_pdl(imp_kernel<DENSE>, dim3(ib, L.n_seq), dim3(256), 0, stream, a);
      if (e != cudaSuccess) return e;
    }
    if (!fused) {
      e = launch_pdl(token_kernel<DENSE>, dim3(blocks > 0 ? blocks : 1, L.n_seq), dim3(256), 0, stream, a);
      if (e != cudaSuccess) return e;
    }
  }
  if (C > 0) {
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg = select_cluster_config(attr, C, L.n_seq, stream);
    e = cudaLaunchKernelEx(&cfg, select_cluster_kernel, a, fused);
    if (e != cudaSuccess) return e;
  } else {
    auto selk = select_kernel<DT, D, DENSE>;
    e = ensure_smem(selk, kSelectSmemMax);
    if (e != cudaSuccess) return e;
    e = launch_pdl(selk, dim3(L.n_seq), dim3(1024), small ? sel_smem : 0, stream, a, small);
    if (e != cudaSuccess) return e;
  }
  if (DENSE || n_evict_hint > kInlineEvict) {
    const int items = DENSE ? S_grid : n_evict_hint;
    int blocks = (items + 7) / 8;
    if (blocks > 592) blocks = 592;
    if (blocks < 1) blocks = 1;
    const size_t stage = (size_t)8 * L.Hk * D * sizeof(T);
    if (stage > 96 * 1024) a.vec_ok = 0;
    auto ek = evict_kernel<DT, D, DENSE>;
    if (a.vec_ok) {
      e = ensure_smem(ek, stage);
      if (e != cudaSuccess) return e;
    }
    e = launch_pdl(ek, dim3(blocks, L.n_seq), dim3(256), a.vec_ok ? stage : 0, stream, a);
  }
  return e;
}

template <int DT, int D>
static cudaError_t compress_dt(CompressArgs a, bool dense, int S_grid, int n_evict_hint, cudaStream_t stream) {
  if (dense) return compress_t<DT, D, true>(a, S_grid, n_evict_hint, stream);
  return compress_t<DT, D, false>(a, S_grid, n_evict_hint, stream);
}

cudaError_t launch_compress(const hc_layer& L, const void* q_obs, int64_t qs0, int64_t qs1, int64_t qs2, int tq,
                            int S_dense, const void* sk, const void* sv, const void* skp, int64_t ss0, int64_t ss1,
                            int64_t ss2, const int64_t* spos, void* scratch, int n_evict_hint, cudaStream_t stream) {
  const bool dense = sk != nullptr;
  const int S_grid = dense ? S_dense : L.max_cap;
  const CompressLayout lay = compress_layout(L, S_grid, tq);
  char* base = reinterpret_cast<char*>(scratch);
  CompressArgs a{};
  a.L = L;
  a.q_obs = q_obs;
  a.qs_seq = qs0; a.qs_head = qs1; a.qs_tok = qs2;
  a.tq = tq;
  a.tqmax = tq > 0 ? tq : 1;
  a.S_dense = S_dense;
  a.S_max = S_grid;
  a.max_chunks = (S_grid + 31) / 32;
  a.src_k = sk; a.src_v = sv; a.src_kpre = skp;
  a.ss_seq = ss0; a.ss_head = ss1; a.ss_tok = ss2;
  {
    const int esz = L.dtype == HC_F32 ? 4 : 2;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    a.vec_ok = (!dense || (al(sk) && al(sv) && al(skp) && (ss0 * esz) % 16 == 0 && (ss1 * esz) % 16 == 0 &&
                           (ss2 * esz) % 16 == 0)) ? 1 : 0;
  }
  a.src_pos = spos;
  a.hdr = reinterpret_cast<int*>(base + lay.hdr);
  a.logits = reinterpret_cast<float*>(base + lay.logits);
  a.part = reinterpret_cast<float*>(base + lay.part);
  a.stats = reinterpret_cast<float*>(base + lay.stats);
  a.imp = reinterpret_cast<float*>(base + lay.imp);
  a.tok = reinterpret_cast<float*>(base + lay.tok);
  a.sel = reinterpret_cast<uint8_t*>(base + lay.sel);
  a.keep_src = reinterpret_cast<int*>(base + lay.keep_src);
  a.ev_src = reinterpret_cast<int*>(base + lay.ev_src);
  a.ev_dst = reinterpret_cast<int*>(base + lay.ev_dst);
  a.qb = base + lay.qb;
  a.chunk_len = kScoreCH;
  if (L.dtype == HC_F32 && L.D == 128) return compress_dt<HC_F32, 128>(a, dense, S_grid, n_evict_hint, stream);
  if (L.dtype == HC_F16 && L.D == 128) return compress_dt<HC_F16, 128>(a, dense, S_grid, n_evict_hint, stream);
  if (L.dtype == HC_BF16 && L.D == 128) return compress_dt<HC_BF16, 128>(a, dense, S_grid, n_evict_hint, stream);
  if (L.dtype == HC_F32 && L.D == 64) return compress_dt<HC_F32, 64>(a, dense, S_grid, n_evict_hint, stream);
  if (L.dtype == HC_F16 && L.D == 64) return compress_dt<HC_F16, 64>(a, dense, S_grid, n_evict_hint, stream);
  if (L.dtype == HC_BF16 && L.D == 64) return compress_dt<HC_BF16, 64>(a, dense, S_grid, n_evict_hint, stream);
  return cudaErrorInvalidValue;
}

size_t compress_scratch_bytes(const hc_layer& L, int S_max, int tq) { return compress_layout(L, S_max, tq).total; }

}  // namespace hc
