// Shared device helpers for the hot/cold decode kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/hotcold_b200.h"

namespace hc {

constexpr float kNegInf = -__builtin_huge_valf();
// Logits at or above this value overflow float32 exp (ln(FLT_MAX) rounded up).
constexpr float kExpOverflow = 88.72283935546875f;
// Upper bound on mbarrier polls before a wait gives up and reports HC_DEV_TIMEOUT; each poll
// suspends for at most kPollSuspendNs, so a wait ends within about a second.
constexpr int kMaxPolls = 1 << 20;
constexpr uint32_t kPollSuspendNs = 1000;

// ----------------------------------------------------------------------------------------
// element types
// ----------------------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<HC_F32> {
  using T = float;
  static __device__ __forceinline__ float load(const T* p) { return *p; }
  static __device__ __forceinline__ float to_f(T x) { return x; }
  static __device__ __forceinline__ T from_f(float x) { return x; }
  static __device__ __forceinline__ float round(float x) { return x; }
};
template <> struct Elem<HC_F16> {
  using T = __half;
  static __device__ __forceinline__ float load(const T* p) { return __half2float(*p); }
  static __device__ __forceinline__ float to_f(T x) { return __half2float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};
template <> struct Elem<HC_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float load(const T* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ float to_f(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};

// Unpack a 16-byte vector of elements into floats.
template <int DT>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (DT == HC_F32) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (DT == HC_F16) {
        __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        float2 t = __half22float2(h);
        f[2 * i] = t.x; f[2 * i + 1] = t.y;
      } else {
        __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
        float2 t = __bfloat1622float2(h);
        f[2 * i] = t.x; f[2 * i + 1] = t.y;
      }
    }
  }
}

// Unpack N consecutive elements (N * element size a multiple of 4 bytes, naturally aligned).
template <int DT, int N>
__device__ __forceinline__ void unpack_n(const void* p, float* f) {
  if constexpr (DT == HC_F32) {
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N; i += 4) {
        const float4 x = reinterpret_cast<const float4*>(p)[i / 4];
        f[i] = x.x; f[i + 1] = x.y; f[i + 2] = x.z; f[i + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N; i += 2) {
        const float2 x = reinterpret_cast<const float2*>(p)[i / 2];
        f[i] = x.x; f[i + 1] = x.y;
      }
    }
  } else {
    static_assert(N % 2 == 0, "pairs of 16-bit elements");
    uint32_t w[N / 2];
    if constexpr (N % 4 == 0) {
#pragma unroll
      for (int i = 0; i < N / 2; i += 2) {
        const uint2 x = reinterpret_cast<const uint2*>(p)[i / 2];
        w[i] = x.x; w[i + 1] = x.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < N / 2; ++i) w[i] = reinterpret_cast<const uint32_t*>(p)[i];
    }
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      float2 t;
      if constexpr (DT == HC_F16) t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      else t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      f[2 * i] = t.x; f[2 * i + 1] = t.y;
    }
  }
}

// RoPE on one element pair, rounded like HF's apply_rotary_pos_emb in the model dtype:
// out = round(round(x*c) + round(rot*s)), each product and the sum a separate op.
template <int DT>
__device__ __forceinline__ float rope_elem(float x, float rot, float c, float s) {
  using E = Elem<DT>;
  float a = E::round(__fmul_rn(x, c));
  float b = E::round(__fmul_rn(rot, s));
  return E::round(__fadd_rn(a, b));
}

// cos/sin of HF's LlamaRotaryEmbedding at one position for frequency index i:
// float32 angle inv_freq[i]*float(pos), float32 cos/sin, times attention_scaling,
// rounded to the model dtype.
template <int DT>
__device__ __forceinline__ void rope_cs(float inv_freq, int64_t pos, float scaling, float& c, float& s) {
  float ang = __fmul_rn(inv_freq, (float)pos);
  c = Elem<DT>::round(__fmul_rn(cosf(ang), scaling));
  s = Elem<DT>::round(__fmul_rn(sinf(ang), scaling));
}

// ----------------------------------------------------------------------------------------
// warp / block reductions
// ----------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Exclusive prefix sum of one int per thread over the block; returns the block total.
// `sh` needs blockDim.x/32 + 1 ints. All threads must call.
__device__ __forceinline__ int block_exclusive_scan(int v, int* sh, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) sh[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  int before = (warp > 0 ? sh[warp - 1] : 0) + x - v;
  total = sh[nw - 1];
  __syncthreads();
  return before;
}

// Monotone map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t fkey(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ----------------------------------------------------------------------------------------
// TMA bulk copies (cp.async.bulk, non-tensor) completing on an mbarrier
// ----------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// One bulk global->shared copy of `bytes` (multiple of 16, both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Bulk copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from this CTA's shared
// memory to the same-offset buffer of cluster CTA `rank`, completing on that CTA's mbarrier at
// the offset of `bar` (distributed shared memory through the TMA engine).
__device__ __forceinline__ void bulk_s2cluster(void* buf, uint32_t bytes, uint64_t* bar, uint32_t rank) {
  uint32_t dst, rbar;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(dst) : "r"(smem_u32(buf)), "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(smem_u32(bar)), "r"(rank));
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "r"(smem_u32(buf)), "r"(bytes), "r"(rbar)
               : "memory");
}
// 32-bit load from the same-offset shared memory word of cluster CTA `rank`.
__device__ __forceinline__ int ld_cluster_s32(const int* p, uint32_t rank) {
  uint32_t addr;
  int v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(smem_u32(p)), "r"(rank));
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kPollSuspendNs)
      : "memory");
  return ok != 0;
}
// Bounded wait on phase `parity`. Returns false after kMaxPolls polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kMaxPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ----------------------------------------------------------------------------------------
// cp.async gathers (16-byte chunks through L2), ldmatrix and the m16n8k16 tensor-core MMA
// ----------------------------------------------------------------------------------------
// Copies 16 bytes; with src_bytes = 0 nothing is read and the destination is zero-filled.
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem, int src_bytes) {
  // no memory clobber: ordering against later shared-memory reads comes from cp_async_wait
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem),
               "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
// c += A(16x16, row) * B(16x8, col), fp32 accumulate; A and B both f16 or both bf16.
template <int DT>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (DT == HC_F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// L2 prefetch hints: one line, or a 16-byte aligned range of a multiple of 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes));
}

// ----------------------------------------------------------------------------------------
// TMA tensor loads and the 5th-generation tensor cores (tcgen05, accumulators in TMEM)
// ----------------------------------------------------------------------------------------
// 2-D tiled TMA load of one box into shared memory, completing on an mbarrier. The tensor map
// lives in global memory (written by the host before the launch).
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst_smem)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Fetch a tensor map (in global memory) into the TMA unit's descriptor cache ahead of its first use.
__device__ __forceinline__ void prefetch_tensormap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// TMEM allocation by one full warp; the column address lands in shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzle layout: rows of
// 128 bytes, 8-row atoms of 1024 bytes placed contiguously (stride 1024), atoms 1024-aligned.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1u << 16;                           // leading byte offset (unused by this layout)
  d |= (uint64_t)(1024u >> 4) << 32;                 // stride byte offset: next 8-row atom
  d |= (uint64_t)1u << 46;                           // descriptor version
  d |= (uint64_t)2u << 61;                           // 128-byte swizzle
  return d;
}
// Descriptor of an MN-major operand in the 128-byte swizzle layout: 8-row (K) atoms of 128-byte
// rows holding 64 MN-contiguous elements, 8-row groups 1024 bytes apart (stride byte offset), the
// next 64 elements of MN `lbo` bytes further (leading byte offset); atoms 1024-aligned.
__device__ __forceinline__ uint64_t umma_desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;       // leading byte offset: next 64 MN elements
  d |= (uint64_t)(1024u >> 4) << 32;                 // stride byte offset: next 8 K rows
  d |= (uint64_t)1u << 46;                           // descriptor version
  d |= (uint64_t)2u << 61;                           // 128-byte swizzle
  return d;
}
// D[tmem] (+)= A[smem] . B[smem]^T for kind::f16 (A and B both f16 or both bf16), fp32 accum.
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 TMEM lanes x 8 columns of 32-bit values: this warp's lane quarter, thread = lane.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Thread-block-cluster barrier halves. Every thread of every CTA in the cluster executes both.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Arrival that releases this thread's prior (distributed) shared memory writes to the threads
// that pass the matching cluster_wait.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.aligned;" ::: "memory"); }

__device__ __forceinline__ void set_status(hc_seq_state* st, int bits) {
  if (st) atomicOr(&st->status, bits);
}

// ----------------------------------------------------------------------------------------
// Programmatic dependent launch: let the next kernel in the stream start its prologue,
// and wait for the previous one before touching its outputs.
// ----------------------------------------------------------------------------------------
// Waits for the preceding kernel of the stream, then lets the next one begin launching at once:
// every kernel launched with programmatic serialization starts with this call, so a dependent
// never reads this kernel's results before this kernel has completed.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ----------------------------------------------------------------------------------------
// host: launch with programmatic stream serialization, dtype x head-dim dispatch
// ----------------------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Raise a kernel's dynamic shared memory limit, once per (kernel, device). The cache is keyed
// on the kernel's address: every template instance needs its own attribute.
template <typename K>
inline cudaError_t ensure_smem(K kern, size_t bytes) {
  struct Entry {
    const void* fn;
    unsigned long long devs;
    size_t bytes;
  };
  static Entry cache[256];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  const void* fn = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lock(mu);
  int i = 0;
  for (; i < n; ++i)
    if (cache[i].fn == fn) break;
  if (i < n && (cache[i].devs & bit) && cache[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return e;
  if (i == n && n < 256) cache[n++] = Entry{fn, 0ull, bytes};
  if (i < n) {
    cache[i].devs |= bit;
    cache[i].bytes = bytes;
  }
  return cudaSuccess;
}

#define HC_DISPATCH_DT_D(dtype, D, FN, ...)                                     \
  do {                                                                          \
    if ((dtype) == HC_F32 && (D) == 128) return FN<HC_F32, 128>(__VA_ARGS__);   \
    if ((dtype) == HC_F16 && (D) == 128) return FN<HC_F16, 128>(__VA_ARGS__);   \
    if ((dtype) == HC_BF16 && (D) == 128) return FN<HC_BF16, 128>(__VA_ARGS__); \
    if ((dtype) == HC_F32 && (D) == 64) return FN<HC_F32, 64>(__VA_ARGS__);     \
    if ((dtype) == HC_F16 && (D) == 64) return FN<HC_F16, 64>(__VA_ARGS__);     \
    if ((dtype) == HC_BF16 && (D) == 64) return FN<HC_BF16, 64>(__VA_ARGS__);   \
    return cudaErrorInvalidValue;                                               \
  } while (0)

}  // namespace hc
