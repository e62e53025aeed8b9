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

// Block-wide exclusive scan of one int per thread with a single barrier:
// every warp scans the warp totals itself.  wtot: 32 ints of shared scratch
// that no other scan uses between this call's barrier and the next one.
__device__ __forceinline__ int block_exclusive_scan_1b(int v, int* total, int* wtot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (int)(blockDim.x >> 5);
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  __syncthreads();
  int t = lane < nw ? wtot[lane] : 0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, t, o);
    if (lane >= o) t += y;
  }
  const int warp_before = __shfl_sync(0xffffffffu, t, warp > 0 ? warp - 1 : 0);
  *total = __shfl_sync(0xffffffffu, t, nw - 1);
  return (warp > 0 ? warp_before : 0) + x - v;
}

// Scratch of block_select_reg (caller's shared memory, 16-byte aligned).
struct RegSelectSmem {
  int hists[3][256];  // digit histograms, rotating by pass
  uint32_t s_or[32], s_and[32];
  int wtot[2][32];    // warp totals of the caller's two scans
};

// The threshold of a top-k selection, the same in every thread: the selection
// is every key greater than thr plus the first take_eq (in index order) of the
// keys equal to it; split is false when every key equal to thr is selected.
struct RegSelection {
  uint32_t thr;
  int take_eq;
  bool split;
};

// The k largest of n keys (1 <= k <= n) held in registers, key[0, cnt) by each
// thread: the same digits, passes and threshold as block_radix_select, with
// one barrier per pass.  The caller has zeroed S.hists[0] and S.hists[1] and
// passes the OR and AND of all n keys (o, a), the same in every thread, both
// before a barrier.  Every warp reads the whole histogram after the pass's
// barrier and finds the threshold bin itself (nothing is broadcast through
// shared memory); the histograms rotate over three buffers, and the one
// cleared after pass r's barrier was last read before that barrier and is
// next filled after pass r + 1's.
template <int KPT>
__device__ __forceinline__ RegSelection block_select_reg(const uint32_t (&key)[KPT], int cnt, int n, int k,
                                                         uint32_t o, uint32_t a, RegSelectSmem& S) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int start = 32 - __clz(o ^ a);  // low bits that differ somewhere; 0: all keys equal
  uint32_t mask = start >= 32 ? 0u : (0xffffffffu << start);
  uint32_t prefix = a & mask;
  int need = k, bin_count = start == 0 ? n : -1;
  int pass = 0;
  for (int shift = start - 8; start > 0; shift -= 8, ++pass) {
    const int sh = max(shift, 0);  // a last digit narrower than 8 bits overlaps fixed bits (constant)
    int* hist = S.hists[pass % 3];
#pragma unroll
    for (int u = 0; u < KPT; ++u)  // plain atomics: faster here than warp-aggregated ones (match.any)
      if (u < cnt && (key[u] & mask) == prefix) atomicAdd(&hist[(key[u] >> sh) & 255u], 1);
    __syncthreads();
    int* next = S.hists[(pass + 2) % 3];
    for (int i = tid; i < 256; i += (int)blockDim.x) next[i] = 0;
    // lane l: bins 255 - 8l - e, e = 0..7 (descending), two 16-byte loads
    const int4 h0 = *reinterpret_cast<const int4*>(hist + 248 - 8 * lane);
    const int4 h1 = *reinterpret_cast<const int4*>(hist + 252 - 8 * lane);
    const int c[8] = {h1.w, h1.z, h1.y, h1.x, h0.w, h0.z, h0.y, h0.x};
    int loc = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) loc += c[e];
    int incl = loc;
#pragma unroll
    for (int w = 1; w < 32; w <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, w);
      if (lane >= w) incl += y;
    }
    const int excl = incl - loc;
    const unsigned hit = __ballot_sync(0xffffffffu, excl < need && need <= incl);
    const int src = hit ? __ffs(hit) - 1 : 0;  // the one lane whose bins hold the need-th key
    int nbin = 0, nneed = need, ncount = 0;
    if (lane == src) {
      int run = excl;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (run < need && need <= run + c[e]) {
          nbin = 255 - 8 * lane - e;
          nneed = need - run;
          ncount = c[e];
        }
        run += c[e];
      }
    }
    nbin = __shfl_sync(0xffffffffu, nbin, src);
    need = __shfl_sync(0xffffffffu, nneed, src);
    bin_count = __shfl_sync(0xffffffffu, ncount, src);
    prefix = (prefix & ~(255u << sh)) | ((uint32_t)nbin << sh);
    mask |= 255u << sh;
    // once the whole threshold bin is needed, every key with this prefix is
    // selected and the lower bits do not matter
    if (sh == 0 || need == bin_count) break;
  }
  return RegSelection{prefix, need, need != bin_count};
}

}  // namespace nsm
