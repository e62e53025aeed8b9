// nsm_common.cuh -- device helpers shared by the sparse NF4 decode kernels.
//
// Dequantization scheme (all batch-1 GEMV kernels):
//   * A per-CTA shared-memory lookup table maps one packed NF4 byte (two
//     nibbles = two consecutive elements, high nibble = even element) to a
//     half2 {code[hi], code[lo]}.  Each entry is replicated once per lane
//     (entry e for lane l at word e*64 + table*32 + l), so a warp-wide lookup
//     of 32 arbitrary bytes hits 32 distinct banks.
//   * The lookup address e*256 + lane*4 is built by ONE byte-permute (prmt)
//     from the packed word and a per-lane constant.
//   * The dequantized fp16 pairs are fed as the A fragment of
//     mma.sync.m16n8k16 (f16 x f16 -> f32); the activation (x, or SiLU*up)
//     is the B fragment (column 0 = the token).  The tensor pipe is used as
//     an fp32-accumulating dot-product engine: the kernels are HBM-bound, the
//     MMA keeps the issue cost per weight low and the accumulation exact
//     (fp16 x fp16 products are exact in fp32).
//   * The reduction index k is permuted so that lane t of a quad owns a
//     contiguous 8-byte (gate/up: 16 columns) or 4-byte (down: 8 columns)
//     run of each row; activations are read in natural order.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/nsm.h"

namespace nsm {

constexpr int kBlock = 32;     // rows (neurons) per intermediate block
constexpr int kQbs = 64;       // NF4 quant block size (absmax group)
constexpr int kLutWordsPerEntry = 64;   // 2 tables x 32 lanes
constexpr int kLutBytes = 256 * kLutWordsPerEntry * 4;  // 64 KB

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == NSM_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == NSM_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_from_f32(void* p, int dtype, int64_t i, float v) {
  if (dtype == NSM_F32) {
    reinterpret_cast<float*>(p)[i] = v;
  } else if (dtype == NSM_F16) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  } else {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
}

// Streaming (read-once) loads: bypass L1 allocation, ask L2 for 256-byte fetches.
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ float4 ldg_f4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ uint32_t ldg_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L2::128B.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ float ldg_f32(const float* p) { return __ldg(p); }
__device__ __forceinline__ uint4 ldg_u4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Bulk prefetch of [p, p + bytes) into L2 (no registers, no shared memory).
// p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- bulk async copies (TMA engine, no multicast) + mbarriers --------------
// A warp streams its weight tiles global -> shared with cp.async.bulk; each
// ring stage has one mbarrier that completes when the stage's bytes landed.
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the async proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Orders this thread's earlier shared-memory accesses (generic proxy) before
// its later bulk copies into shared memory (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Evict-first L2 policy for bytes that are read exactly once.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Evict-last L2 policy for small vectors that every CTA copies.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Orders global writes of earlier kernels / other threads (generic proxy),
// acquired by this thread, before its later bulk copies from global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// global -> shared bulk copy (16-byte aligned addresses, size a multiple of
// 16); completion is counted on mbarrier `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(pol)
      : "memory");
}
// Bounded wait for phase `parity` of mbarrier `bar`; false when the bound ran
// out (the caller records an error instead of spinning forever).  The kernels
// take the bound of their first waits from their launch parameters (the
// process-wide setting of nsm_set_copy_wait_limit); waits that drain a ring
// after a failure always use the default bound, so a warp never leaves
// while copies into its shared memory are still in flight.
constexpr int kMbarSpinLimit = 1 << 22;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int limit = kMbarSpinLimit) {
  for (int i = 0; i < limit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred P;\n mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n selp.u32 %0, 1, 0, P;\n}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}
__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}
__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 r;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "r"(addr));
  return r;
}

// 8-byte system-scope relaxed store / load: a value and its epoch travel in one
// single-copy-atomic word between GPUs.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Loads of data written by other CTAs of the same kernel (skip L1).
__device__ __forceinline__ float ldcg_f32(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int ldcg_i32(const int* p) { return __ldcg(p); }
__device__ __forceinline__ uint32_t ldcg_u32(const uint32_t* p) { return __ldcg(p); }

// Fill the per-lane-replicated byte->half2 tables from up to two 16-entry
// fp32 codebooks.  Table t at word e*64 + t*32 + lane.
__device__ __forceinline__ void build_lut(uint32_t* lut, const float* code0, const float* code1) {
  __shared__ uint32_t pairs[2][256];
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int t = i >> 8, e = i & 255;
    const float* c = t == 0 ? code0 : code1;
    __half lo = __float2half_rn(c[e >> 4]);
    __half hi = __float2half_rn(c[e & 15]);
    pairs[t][e] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
  }
  __syncthreads();
  uint4* lut4 = reinterpret_cast<uint4*>(lut);
  for (int i = threadIdx.x; i < 256 * kLutWordsPerEntry / 4; i += blockDim.x) {
    const int e = i >> 4;            // 16 uint4 per entry
    const int t = (i >> 3) & 1;      // 8 uint4 per table-row of 32 words
    const uint32_t v = pairs[t][e];
    lut4[i] = make_uint4(v, v, v, v);
  }
  __syncthreads();
}

// Table lookup of byte `sel` (0..3) of `w`: half2 {code[hi nibble], code[lo nibble]}.
template <int kByte, int kTable>
__device__ __forceinline__ uint32_t lut_lookup(const uint32_t* lut, uint32_t w, uint32_t lanebase) {
  // address bytes: [lane*4, w.byte[kByte], 0, 0] -> e*256 + lane*4
  const uint32_t addr = __byte_perm(w, lanebase, 0x5504u | (kByte << 4));
  return *reinterpret_cast<const uint32_t*>(reinterpret_cast<const char*>(lut) + addr + kTable * 128);
}

// Same lookup with the byte index and table as (unrolled) values.
__device__ __forceinline__ uint32_t lut_lookup_rt(const uint32_t* lut, uint32_t w, uint32_t lanebase, int kbyte,
                                                  int table) {
  const uint32_t addr = __byte_perm(w, lanebase, 0x5504u | ((uint32_t)kbyte << 4));
  return *reinterpret_cast<const uint32_t*>(reinterpret_cast<const char*>(lut) + addr + table * 128);
}

// (not volatile: a pure register computation the compiler may schedule freely)
__device__ __forceinline__ void mma_16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Power-of-two scale s = 2^e with max|v|/s in [2^14, 2^15); 1 for an all-zero run.
__device__ __forceinline__ float pow2_scale_for(float maxabs) {
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 1.f;
  int e = ilogbf(maxabs) - 14;
  return ldexpf(1.f, e);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait (no-op without the launch attribute) until the previous
// kernel has completed and its writes are visible.
// ---- balanced work streams ---------------------------------------------------
// Both gather-GEMVs split their (block, tile) pairs into `nw` contiguous,
// equal ranges, one per warp (sizes differ by at most one pair), so every warp
// finishes at the same time and its load pipeline never restarts at a block
// boundary.  A warp flushes its fp32 accumulators whenever its range crosses
// the boundary of a reduction group (a block for gate/up, a row group for
// down); the segments of one group are reduced in fixed order by the
// finalize kernels, so results are deterministic.
__device__ __forceinline__ int stream_begin(int total, int nw, int w) {
  return (int)(((long long)total * w) / nw);
}
// The warp whose range holds pair x: the largest w with stream_begin(w) <= x.
__device__ __forceinline__ int stream_owner(int total, int nw, int x) {
  return (int)((((long long)x + 1) * nw - 1) / total);
}
// Warps for `groups` reduction groups of `len` pairs with at most `max_seg`
// segments per group: every range holds >= ceil(len / (max_seg - 2)) pairs.
__device__ __forceinline__ int stream_warps(int groups, int len, int max_seg, int total_warps) {
  const int total = groups * len;
  const int m = max(1, (len + max_seg - 3) / (max_seg - 2));
  return max(1, min(total_warps, total / m));
}

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float silu_f32(float g) { return g / (1.f + expf(-g)); }

}  // namespace nsm
