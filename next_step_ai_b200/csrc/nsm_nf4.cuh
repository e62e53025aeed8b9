// nsm_nf4.cuh -- NF4 dequantisation tables and the mma.sync dot engine shared by
// the decode kernels (nsm_decode.cu) and the multi-token union kernels
// (nsm_union.cu).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "nsm_common.cuh"

namespace nsm {

// Dynamic shared memory of both MLP kernels: [0, 64 KB) byte->half2 tables,
// then 2 KB of table-building scratch, then per-call vectors staged once per
// CTA (x16 + xscale for gate/up; act16 + act_scale + rows for down).
extern __shared__ __align__(1024) uint32_t g_lut_smem[];
constexpr int kLutScratch = 2048;
constexpr int kSmemHead = kLutBytes + kLutScratch;

// Byte `kbyte` of w -> half2 from table `table`.  One byte-permute builds
// the table-relative address e*256 + lane*4; kBase >= 0 is the shared-window
// address of the table, folded into the load's immediate offset (the user
// shared memory of a CTA starts after a reserved 1 KB, so the base is 0x400
// when the kernel has no static shared variables).  kBase < 0: generic path.
template <int kBase>
__device__ __forceinline__ uint32_t lut_get(uint32_t w, uint32_t lanebase, int kbyte, int table) {
  const uint32_t addr = __byte_perm(w, lanebase, 0x5504u | ((uint32_t)kbyte << 4));
  if (kBase >= 0) {
    // not volatile: the tables are constant after the prologue's barrier and
    // the address depends on weight bytes loaded after it, so the compiler may
    // interleave these loads with independent MMA chains
    uint32_t v;
    if (table == 0)
      asm("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(kBase));
    else
      asm("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(kBase + 128));
    return v;
  } else {
    return *reinterpret_cast<const uint32_t*>(reinterpret_cast<const char*>(g_lut_smem) + addr + table * 128);
  }
}

__device__ __forceinline__ uint32_t lut_base_addr() { return (uint32_t)__cvta_generic_to_shared(g_lut_smem); }

__device__ __forceinline__ void mma_16816_z(float d[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                            uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

__device__ __forceinline__ void build_lut_dyn(const float* code0, const float* code1) {
  uint32_t* pairs = g_lut_smem + kLutBytes / 4;  // scratch [2][256]
  for (int i = threadIdx.x; i < 512; i += blockDim.x) {
    const int t = i >> 8, e = i & 255;
    const float* c = t == 0 ? code0 : code1;
    const __half lo = __float2half_rn(c[e >> 4]);
    const __half hi = __float2half_rn(c[e & 15]);
    pairs[i] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
  }
  __syncthreads();
  uint4* lut4 = reinterpret_cast<uint4*>(g_lut_smem);
  for (int i = threadIdx.x; i < 256 * kLutWordsPerEntry / 4; i += blockDim.x) {
    const uint32_t v = pairs[((i >> 3) & 1) * 256 + (i >> 4)];
    lut4[i] = make_uint4(v, v, v, v);
  }
}

}  // namespace nsm
