// nsm_select.cuh -- block-wide exact top-k selection over order-preserving
// float keys in shared memory, shared by the router's top-k kernel and the
// gate/up kernel (which selects the blocks itself on the decode path).
//
// Nothing here declares static shared memory: the scratch comes from the
// caller (the gate/up kernel keeps its lookup table at the start of dynamic
// shared memory).
#pragma once

#include <stdint.h>

#include "nsm_common.cuh"

namespace nsm {

// Float -> unsigned key with the same order (larger float, larger key).
__device__ __forceinline__ uint32_t orderable(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_orderable(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// Block-wide exclusive scan of one int per thread (blockDim <= 1024, a
// multiple of 32); wsum: 32 ints of shared scratch.
__device__ __forceinline__ int block_exclusive_scan_s(int v, int* total, int* wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < nw ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) wsum[lane] = s;  // inclusive
  }
  __syncthreads();
  const int before = (warp > 0 ? wsum[warp - 1] : 0) + x - v;
  *total = wsum[nw - 1];
  __syncthreads();
  return before;
}

// Shared state and scratch of block_radix_select.
struct RadixSelectSmem {
  int hists[2][256];  // digit histograms, alternating by pass
  uint32_t s_or[32], s_and[32];
  int wsum[32];       // scan scratch for the caller
  uint32_t prefix, mask;
  int need, bin_count, start;
};

// The k largest of the n keys in shared memory (1 <= k <= n), by the whole
// CTA: the keys' common leading bits are skipped (kor / kand: OR / AND of the
// keys this thread loaded), then 8-bit digits from the top with
// warp-aggregated histogram increments; a pass stops once the whole threshold
// bin is needed.  On return (every thread): the selection is every key
// greater than S.prefix plus the first S.need (in index order) of the keys
// equal to it; S.need == S.bin_count when no tie is split, and then every key
// >= S.prefix is selected.
__device__ __forceinline__ void block_radix_select(const uint32_t* keys, int n, int k, uint32_t kor, uint32_t kand,
                                                   RadixSelectSmem& S) {
  const int tid = threadIdx.x;
  for (int i = tid; i < 512; i += blockDim.x) (&S.hists[0][0])[i] = 0;
  kor = __reduce_or_sync(0xffffffffu, kor);
  kand = __reduce_and_sync(0xffffffffu, kand);
  if ((tid & 31) == 0) {
    S.s_or[tid >> 5] = kor;
    S.s_and[tid >> 5] = kand;
  }
  __syncthreads();
  if (tid < 32) {
    const int nwarps = (int)(blockDim.x >> 5);
    const uint32_t o = __reduce_or_sync(0xffffffffu, tid < nwarps ? S.s_or[tid] : 0u);
    const uint32_t a = __reduce_and_sync(0xffffffffu, tid < nwarps ? S.s_and[tid] : 0xffffffffu);
    if (tid == 0) {
      const int start = 32 - __clz(o ^ a);  // low bits that differ somewhere; 0: all keys equal
      const uint32_t hi = start >= 32 ? 0u : (0xffffffffu << start);
      S.prefix = a & hi;
      S.mask = hi;
      S.need = k;
      S.bin_count = start == 0 ? n : -1;
      S.start = start;
    }
  }
  __syncthreads();
  const int start = S.start;
  int pass = 0;
  for (int shift = start - 8; start > 0; shift -= 8, ++pass) {
    const int sh = max(shift, 0);  // a last digit narrower than 8 bits overlaps fixed bits (constant)
    int* hist = S.hists[pass & 1];  // zero: cleared above / during the previous pass's scan
    const uint32_t pre = S.prefix, msk = S.mask;
    for (int i0 = 0; i0 < n; i0 += blockDim.x) {
      const int i = i0 + tid;
      const uint32_t key = i < n ? keys[i] : 0u;
      const bool on = i < n && (key & msk) == pre;
      const uint32_t bin = on ? ((key >> sh) & 255u) : 256u;
      const unsigned grp = __match_any_sync(0xffffffffu, bin);
      if (on && (threadIdx.x & 31) == (__ffs(grp) - 1)) atomicAdd(&hist[bin], __popc(grp));
    }
    __syncthreads();
    if (tid < 32) {
      // lane l owns bins [255-8l-7, 255-8l] (descending)
      int c[8];
      int loc = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = hist[255 - 8 * tid - e];
        loc += c[e];
      }
      int incl = loc;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += y;
      }
      const int excl = incl - loc;
      const int need = S.need;
      if (excl < need && need <= incl) {
        int run = excl;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (run < need && need <= run + c[e]) {
            const uint32_t bin = 255u - 8u * tid - e;
            S.prefix = (pre & ~(255u << sh)) | (bin << sh);
            S.mask = msk | (255u << sh);
            S.need = need - run;
            S.bin_count = c[e];  // after the last pass: keys equal to the threshold
          }
          run += c[e];
        }
      }
    } else {
      // the next pass's histogram is cleared while warp 0 scans this one
      for (int i = tid - 32; i < 256; i += (int)blockDim.x - 32) S.hists[(pass + 1) & 1][i] = 0;
    }
    __syncthreads();
    // once the whole threshold bin is needed, every key with this prefix is
    // selected and the lower bits do not matter
    if (sh == 0 || S.need == S.bin_count) break;
  }
}

}  // namespace nsm
