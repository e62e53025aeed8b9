// nsm_nf4.cuh -- NF4 dequantisation tables and the mma.sync dot engine shared by
// the decode kernels (nsm_decode.cu) and the multi-token union kernels
// (nsm_union.cu).
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "nsm_common.cuh"

namespace nsm {

// Dynamic shared memory of both MLP kernels: [0, 64 KB) byte->half2 tables,
// then 2 KB of table-building scratch and 256 B holding the tables' codebook
// prescales, then per-call vectors staged once per CTA (x16 + xscale for
// gate/up; act16 + act_scale + rows for down).
extern __shared__ __align__(1024) uint32_t g_lut_smem[];
constexpr int kLutScratch = 2048 + 256;
constexpr int kSmemHead = kLutBytes + kLutScratch;
constexpr int kLutAlphaOff = kLutBytes + 2048;  // float alpha[2], inv_alpha[2]

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

__device__ __forceinline__ float* lut_alpha_smem() {
  return reinterpret_cast<float*>(reinterpret_cast<char*>(g_lut_smem) + kLutAlphaOff);
}
// 1 / alpha of table t (valid after build_lut_alpha and a barrier)
__device__ __forceinline__ float lut_inv_alpha(int t) { return lut_alpha_smem()[2 + t]; }

// Tables with prescaled codebooks: table t holds {fp16(a_t * code[hi]),
// fp16(a_t * code[lo])} per packed byte, where a_t in [1, 2) (256 candidates,
// step 1/256) minimises sum_k (fp16(a * c_k) * (1 / a) - c_k)^2, ties to the
// smaller a.  fp16 keeps 11 significant bits, so the scaled codebook sits
// closer to representable values than the raw one; the consumer multiplies its
// dot products by 1 / a_t (lut_inv_alpha).  Thread i of the CTA scores
// candidates i, i + blockDim.x, ... of the 512 (two tables x 256); the best of
// each 32-candidate chunk goes to the pair scratch, then warps 0 and 1 reduce
// the chunks of tables 0 and 1.  Every thread of the CTA (at least 64) takes part.
// both = false: table 0 only (code1 is ignored, the second table's words are
// left untouched and lut_inv_alpha(1) reads table 0's).
__device__ __forceinline__ void build_lut_alpha(const float* code0, const float* code1, bool both = true) {
  float* al = lut_alpha_smem();
  float* werr = reinterpret_cast<float*>(g_lut_smem + kLutBytes / 4);  // [2][32] best error per chunk
  int* widx = reinterpret_cast<int*>(werr + 64);                      // [2][32] its candidate
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 64; i += blockDim.x) {
    werr[i] = 3.0e38f;
    widx[i] = 256;
  }
  __syncthreads();
  const int ncand = both ? 512 : 256;
  for (int i0 = 0; i0 < ncand; i0 += (int)blockDim.x) {
    const int i = i0 + (int)threadIdx.x;
    const int t = (i >> 8) & 1, ci = i & 255;
    const float* c = t == 0 ? code0 : code1;
    const float a = 1.f + (float)ci * (1.f / 256.f);
    const float ia = 1.f / a;
    float e = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float ck = __ldg(c + k);
      const float d = __half2float(__float2half_rn(a * ck)) * ia - ck;
      e = fmaf(d, d, e);
    }
    if (i >= ncand) e = 3.0e38f;
    // best (smallest error, then smallest candidate) of the warp's 32; a warp
    // covers one table (32 divides 256)
    int bi = ci;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oe = __shfl_xor_sync(0xffffffffu, e, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oe < e || (oe == e && oi < bi)) {
        e = oe;
        bi = oi;
      }
    }
    if (lane == 0 && i < ncand) {  // one slot per 32-candidate chunk of a table
      werr[t * 32 + (ci >> 5)] = e;
      widx[t * 32 + (ci >> 5)] = bi;
    }
  }
  __syncthreads();
  if (warp < (both ? 2 : 1)) {
    float e = werr[warp * 32 + lane];
    int bi = widx[warp * 32 + lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oe = __shfl_xor_sync(0xffffffffu, e, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oe < e || (oe == e && oi < bi)) {
        e = oe;
        bi = oi;
      }
    }
    if (lane == 0) {
      const float a = 1.f + (float)bi * (1.f / 256.f);
      al[warp] = a;
      al[2 + warp] = 1.f / a;
      if (!both) {
        al[1] = a;
        al[3] = 1.f / a;
      }
    }
  }
  __syncthreads();
  uint32_t* pairs = g_lut_smem + kLutBytes / 4;  // scratch [2][256]
  for (int i = threadIdx.x; i < ncand; i += blockDim.x) {
    const int t = i >> 8, e = i & 255;
    const float* c = t == 0 ? code0 : code1;
    const float a = al[t];
    const __half lo = __float2half_rn(a * __ldg(c + (e >> 4)));
    const __half hi = __float2half_rn(a * __ldg(c + (e & 15)));
    pairs[i] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
  }
  __syncthreads();
  uint4* lut4 = reinterpret_cast<uint4*>(g_lut_smem);
  for (int i = threadIdx.x; i < 256 * kLutWordsPerEntry / 4; i += blockDim.x) {
    if (!both && ((i >> 3) & 1)) continue;
    const uint32_t v = pairs[((i >> 3) & 1) * 256 + (i >> 4)];
    lut4[i] = make_uint4(v, v, v, v);
  }
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
