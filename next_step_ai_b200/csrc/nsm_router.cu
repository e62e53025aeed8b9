// nsm_router.cu -- learned-basis router on sm_100a (one token, or many rows).
//
// router_latent_kernel (split-H, ~128 columns per CTA):
//   * x preparation: the residual += the previous layer's output (its pending
//     down partials summed here, and with several GPUs exchanged over NVLink),
//     RMSNorm sum of squares, fp16 copy of the MLP input with one power-of-two
//     scale per 64 columns (consumed by the gate/up kernel);
//   * partial latent = enc_w[:, slice] . x[slice] with 16-byte loads of enc_w
//     issued before x is ready (multi-row routing: up to 32 rows per CTA);
//   * x-prep-only launches (the final residual flush): the last CTA (atomic
//     ticket) reduces the partials.
// router_scores_kernel:
//   * every CTA reduces the partial latents in fixed order, applies the
//     RMSNorm scale, enc_b and the optional basis top-k mask
//     (streaming_llama_runtime.py:4220-4238);
//   * one thread per block: score = clamp0(latent . score_w[b] + score_b[b])
//     (or |latent| . dec_norm_t[:, b] in legacy mode), times down_block_norm.
// router_topk_kernel:
//   * one 1024-thread CTA per row selects the top-k with an 8-bit-digit radix
//     select on order-preserving score bits (the keys' common leading bits
//     skipped), resolves ties at the threshold by lower block id, orders the
//     k winners (score desc, block id asc) when asked, and compacts them into
//     pool rows through the block map (:4324-4352).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <type_traits>

#include "nsm_common.cuh"
#include "nsm_internal.h"
#include "nsm_router.h"
#include "nsm_select.cuh"

namespace nsm {

template <typename T>
struct Vec8;  // 8 elements from one 16-byte load (T = bf16/f16) or two (f32)
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float v[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <>
struct Vec8<__half> {
  static __device__ __forceinline__ void load(const __half* p, float v[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float v[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
};

// ---------------------------------------------------------------------------
// router A
// ---------------------------------------------------------------------------
// The previous layer's output for columns [c0, c0+n): fixed-order sum of the
// down kernel's segments (the down launch records its warp count and row-group
// size in ws.down_meta; the segment arithmetic mirrors the down kernels').
__device__ __forceinline__ void pending_output(const RouterAParams& p, int c0, int n, float* ybuf) {
  if (n <= (int)blockDim.x) {
    // one column per thread: every segment's word is requested together with
    // the selection count and the down launch's shape (one round trip); the
    // segments past this group's count are ignored
    const int i = threadIdx.x, c = c0 + i;
    const int count = ldcg_i32(p.ws.count);
    const int nw_down = ldcg_i32(p.ws.down_meta), glog = ldcg_i32(p.ws.down_meta + 1);
    float v[kMaxSlotGroups];
#pragma unroll
    for (int q = 0; q < kMaxSlotGroups; ++q) v[q] = i < n ? ldcg_f32(p.ws.ypart + (int64_t)q * p.H + c) : 0.f;
    if (i < n) {
      float y = 0.f;
      if (count > 0 && nw_down > 0) {
        const int G = p.H >> glog, g = c >> glog, total = G * count;
        const int nw = stream_warps(G, count, kMaxSlotGroups, nw_down);
        const int nseg = stream_owner(total, nw, g * count + count - 1) - stream_owner(total, nw, g * count) + 1;
#pragma unroll
        for (int q = 0; q < kMaxSlotGroups; ++q)
          if (q < nseg) y += v[q];
      }
      ybuf[i] = y;
    }
    __syncthreads();
    return;
  }
  const int count = ldcg_i32(p.ws.count);
  const int nw_down = ldcg_i32(p.ws.down_meta), glog = ldcg_i32(p.ws.down_meta + 1);
  const int G = p.H >> glog;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int c = c0 + i;
    float y = 0.f;
    if (count > 0 && nw_down > 0) {
      const int g = c >> glog, total = G * count;
      const int nw = stream_warps(G, count, kMaxSlotGroups, nw_down);
      const int nseg = stream_owner(total, nw, g * count + count - 1) - stream_owner(total, nw, g * count) + 1;
      // 16 segment loads in flight at a time, summed in fixed order
      for (int q0 = 0; q0 < nseg; q0 += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u)
          v[u] = q0 + u < nseg ? ldcg_f32(p.ws.ypart + (int64_t)(q0 + u) * p.H + c) : 0.f;
#pragma unroll
        for (int u = 0; u < 16; ++u) y += v[u];
      }
    }
    ybuf[i] = y;
  }
  __syncthreads();
}

// Cross-GPU sum of this CTA's chunk.  Every value travels with its epoch in one
// 8-byte store (value bits | epoch << 32), so a receiver polls the words
// themselves -- no fences and no separate flag round trip: rank r stores its
// chunk into every rank's buffer (slot epoch & 1, row r); each thread then
// waits (bounded) until its columns carry the current epoch from every rank
// and sums them in rank order -- identical bits on every rank.
__device__ __forceinline__ void exchange_chunk(const RouterAParams& p, int c0, int n, float* ybuf, uint32_t epoch) {
  const ExchangeDev& ex = p.ex;
  const int slot = (int)(epoch & 1u);
  for (int r = 0; r < ex.world; ++r) {
    unsigned long long* dst = ex.data[r] + ((int64_t)slot * ex.world + ex.rank) * ex.hidden + c0;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      st_relaxed_sys_u64(dst + i, (unsigned long long)__float_as_uint(ybuf[i]) | ((unsigned long long)epoch << 32));
  }
  const unsigned long long* src = ex.data[ex.rank] + (int64_t)slot * ex.world * ex.hidden + c0;
  bool timed_out = false;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float y = 0.f;
    for (int r = 0; r < ex.world; ++r) {
      const unsigned long long* w = src + (int64_t)r * ex.hidden + i;
      unsigned long long v = ld_relaxed_sys_u64(w);
      int it = 0;
      while ((uint32_t)(v >> 32) != epoch && !timed_out) {
        if (++it >= ex.spin_limit) {
          timed_out = true;
          break;
        }
        v = ld_relaxed_sys_u64(w);
      }
      y += __uint_as_float((uint32_t)v);
    }
    ybuf[i] = y;
  }
  if (timed_out) atomicCAS(p.ws.err, 0, NSM_ERR_TIMEOUT);
  __syncthreads();
}

constexpr int kLatentRowsPerCta = 32;

template <typename WT>
__global__ void __launch_bounds__(256, 1) router_latent_kernel(RouterAParams p) {
  extern __shared__ float xs[];  // [cols_per_cta] x slice | [cols_per_cta] pending output
  __shared__ float red[8];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * p.cols_per_cta;
  const int c1 = min(p.H, c0 + p.cols_per_cta);
  const int n = c1 - c0;  // multiple of 64
  const WT* enc = reinterpret_cast<const WT*>(p.enc_w);

  // encoder rows for this slice: issue the loads before x is ready
  // (fast path: rank <= 64 and 32 columns per thread of 2-byte weights)
  const int seg = n >> 2;  // multiple of 16
  const bool fast = enc != nullptr && p.rank <= 64 && seg == 32 && sizeof(WT) == 2;
  uint4 pre[4];
  if (fast) {
    const int r = tid >> 2, q = tid & 3;
    if (r < p.rank) {
      const uint4* row = reinterpret_cast<const uint4*>(enc + (int64_t)r * p.H + c0 + q * seg);
#pragma unroll
      for (int i = 0; i < 4; ++i) pre[i] = __ldg(row + i);
    }
  }
  // this thread's RMSNorm weight (a layer weight, not written upstream)
  const bool one_col = !p.multi_rows && n <= (int)blockDim.x;  // one column per thread (always, H <= 65536)
  float nwv = 1.f;
  if (one_col && tid < n && p.residual != nullptr && p.norm_w != nullptr)
    nwv = load_as_f32(p.norm_w, p.norm_w_dtype, c0 + tid);
  pdl_trigger();
  pdl_wait();  // residual / x / y_prev come from earlier kernels
  // the residual load goes out together with the pending-output loads
  float res = 0.f;
  if (one_col && tid < n && p.residual != nullptr) res = p.residual[c0 + tid];
  float* ybuf = xs + p.cols_per_cta;  // [cols_per_cta]: the pending output of the previous layer
  uint32_t epoch = 0;
  if (p.pending) {
    pending_output(p, c0, n, ybuf);
    if (p.ex.world > 1) {
      epoch = ldcg_u32(p.ex.counter) + 1u;
      exchange_chunk(p, c0, n, ybuf, epoch);
    }
  }
  // rows of x this CTA handles: one, or (multi-row routing) up to
  // kLatentRowsPerCta, whose slices are loaded together and then multiplied
  // by the encoder slice held in registers, one row after the other
  const int row0 = p.multi_rows ? blockIdx.y * kLatentRowsPerCta : 0;
  const int row1 = p.multi_rows ? min(p.multi_rows, row0 + kLatentRowsPerCta) : 1;
  if (p.multi_rows) {
    const int total = (row1 - row0) * n;
    for (int i0 = 0; i0 < total; i0 += 16 * (int)blockDim.x) {
      float v[16];  // 16 loads in flight per thread
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int i = i0 + u * (int)blockDim.x + tid, rr = i / n;
        v[u] = i < total ? load_as_f32(p.x, p.x_dtype, (int64_t)(row0 + rr) * p.H + c0 + (i - rr * n)) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int i = i0 + u * (int)blockDim.x + tid;
        if (i < total) xs[i] = v[u];
      }
    }
    __syncthreads();
  }
  for (int row = row0; row < row1; ++row) {
    const float* xr = xs + (row - row0) * n;  // this row's slice
    if (!p.multi_rows) {
      float sumsq = 0.f;
      for (int i = tid; i < n; i += blockDim.x) {
        const int c = c0 + i;
        float v;
        if (p.residual != nullptr) {
          v = one_col ? res : p.residual[c];
          if (p.pending) v += ybuf[i];
          else if (p.y_prev != nullptr) v += load_as_f32(p.y_prev, p.y_prev_dtype, c);
          p.residual[c] = v;
          sumsq += v * v;
          if (p.norm_w != nullptr) v *= one_col ? nwv : load_as_f32(p.norm_w, p.norm_w_dtype, c);
        } else {
          v = load_as_f32(p.x, p.x_dtype, (int64_t)row * p.H + c);
        }
        xs[i] = v;
      }
      sumsq = warp_sum(sumsq);
      if (lane == 0) red[warp] = sumsq;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < 8; ++w) t += red[w];
        p.ws.sumsq_part[row * kRouterMaxCtas + blockIdx.x] = t;
      }
      for (int tl = warp; tl < (n >> 6); tl += 8) {
        const float a = xs[tl * 64 + lane], b = xs[tl * 64 + 32 + lane];
        const float m = warp_max(fmaxf(fabsf(a), fabsf(b)));
        const float s = pow2_scale_for(m);
        const float inv = 1.f / s;
        const int c = c0 + tl * 64;
        // fp16 hi + lo: the gate/up kernels feed both to the tensor cores
        const __half ah = __float2half_rn(a * inv), bh = __float2half_rn(b * inv);
        p.ws.x16[c + lane] = ah;
        p.ws.x16[c + 32 + lane] = bh;
        p.ws.x16lo[c + lane] = __float2half_rn(a * inv - __half2float(ah));
        p.ws.x16lo[c + 32 + lane] = __float2half_rn(b * inv - __half2float(bh));
        if (lane == 0) p.ws.xscale[c >> 6] = s;
      }
    }
    if (fast) {
      const int r = tid >> 2, q = tid & 3;
      float acc = 0.f;
      if (r < p.rank) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w4[4] = {pre[i].x, pre[i].y, pre[i].z, pre[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float lo, hi;
            if (sizeof(WT) == 2 && std::is_same<WT, __half>::value) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
              lo = f.x;
              hi = f.y;
            } else {
              lo = __uint_as_float(w4[e] << 16);
              hi = __uint_as_float(w4[e] & 0xffff0000u);
            }
            acc = fmaf(lo, xr[q * seg + i * 8 + 2 * e], acc);
            acc = fmaf(hi, xr[q * seg + i * 8 + 2 * e + 1], acc);
          }
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (q == 0 && r < p.rank) p.ws.latent_part[((int64_t)row * kRouterMaxCtas + blockIdx.x) * p.rank + r] = acc;
    } else if (enc != nullptr) {
      // thread (row r, quarter q): columns [q*n/4, (q+1)*n/4) of this slice
      for (int r0 = 0; r0 < p.rank; r0 += 64) {
        const int r = r0 + (tid >> 2), q = tid & 3;
        float acc = 0.f;
        if (r < p.rank) {
          const WT* erow = enc + (int64_t)r * p.H + c0 + q * seg;
          for (int i = 0; i < seg; i += 16) {
            float a[8], b[8];
            Vec8<WT>::load(erow + i, a);
            Vec8<WT>::load(erow + i + 8, b);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(a[e], xr[q * seg + i + e], acc);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc = fmaf(b[e], xr[q * seg + i + 8 + e], acc);
          }
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (q == 0 && r < p.rank) p.ws.latent_part[((int64_t)row * kRouterMaxCtas + blockIdx.x) * p.rank + r] = acc;
      }
    }
  }
  if (p.reduce_in_scores) return;  // the scores kernel reduces the partials (and advances the epoch)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(p.ws.ticket_router_a, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __shared__ float s_norm;
  __shared__ float lat[kMaxRank];
  __shared__ float part4[4][kMaxRank];
  const int nparts = gridDim.x;
  if (warp == 0) {
    float t = 0.f;
    if (p.use_norm)
      for (int b = lane; b < nparts; b += 32) t += ldcg_f32(&p.ws.sumsq_part[b]);
    t = warp_sum(t);
    if (lane == 0) {
      const float ns = p.use_norm ? 1.f / sqrtf(t / (float)p.H + p.eps) : 1.f;
      s_norm = ns;
      *p.ws.norm_scale = ns;
    }
  }
  if (enc != nullptr) {
    for (int e = tid; e < 4 * p.rank; e += blockDim.x) {
      const int r = e >> 2, q = e & 3;
      float acc = 0.f;
#pragma unroll 32
      for (int b = q; b < nparts; b += 4) acc += ldcg_f32(&p.ws.latent_part[b * p.rank + r]);
      part4[q][r] = acc;
    }
  }
  __syncthreads();
  if (enc != nullptr) {
    for (int r = tid; r < p.rank; r += blockDim.x) {
      float acc = (part4[0][r] + part4[1][r]) + (part4[2][r] + part4[3][r]);
      acc *= s_norm;
      if (p.enc_b != nullptr) acc += load_as_f32(p.enc_b, p.wdtype, r);
      lat[r] = acc;
    }
    __syncthreads();
    const int bk = max(1, min(p.basis_top_k, p.rank));
    for (int r = tid; r < p.rank; r += blockDim.x) {
      float v = lat[r];
      if (bk < p.rank) {
        const float a = fabsf(v);
        int pos = 0;
        for (int q = 0; q < p.rank; ++q) {
          const float b = fabsf(lat[q]);
          pos += (b > a) || (b == a && q < r);
        }
        if (pos >= bk) v = 0.f;
      }
      p.ws.latent[r] = v;
    }
  }
  if (tid == 0) {
    *p.ws.ticket_router_a = 0;
    if (p.pending && p.ex.world > 1) *p.ex.counter = epoch;  // this rank finished exchange `epoch`
  }
}

// ---------------------------------------------------------------------------
// router B
// ---------------------------------------------------------------------------
__device__ __forceinline__ int map_block(const RouterBParams& p, int b) {
  if (b < 0 || b >= p.NB) return -1;
  int r;
  if (p.slot_of_block != nullptr) {
    r = p.slot_of_block[b];
  } else {
    r = (b >= p.block_begin && b < p.block_end) ? b - p.block_begin : -1;
  }
  return (r >= 0 && r < p.pool_rows) ? r : -1;
}

// Block-wide exclusive scan of one int per thread (blockDim <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int v, int* total) {
  __shared__ int wsum[32];
  return block_exclusive_scan_s(v, total, wsum);
}

// Compacts sel[0..k) through the block map into ws.rows / ws.row_block / ws.count.
__device__ void compact_selection(const RouterBParams& p, const int* sel, int k) {
  __shared__ int s_base;
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  for (int j0 = 0; j0 < k; j0 += blockDim.x) {
    const int j = j0 + threadIdx.x;
    const int r = j < k ? map_block(p, sel[j]) : -1;
    int tot;
    const int pos = block_exclusive_scan(r >= 0 ? 1 : 0, &tot);
    if (r >= 0) {
      p.ws.rows[s_base + pos] = r;
      p.ws.row_block[s_base + pos] = sel[j];
    }
    __syncthreads();
    if (threadIdx.x == 0) s_base += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) *p.ws.count = s_base;
}

template <typename WT>
__device__ __forceinline__ float score_row(const RouterBParams& p, const float* lat, int b) {
  const WT* row = reinterpret_cast<const WT*>(p.score_w) + (int64_t)b * p.rank;
  float acc = 0.f;
  if (p.rank == 64) {
    // all of the row's loads in flight at once
    float v[64];
#pragma unroll
    for (int r = 0; r < 64; r += 8) Vec8<WT>::load(row + r, v + r);
    if (p.legacy) {
#pragma unroll
      for (int r = 0; r < 64; ++r) acc = fmaf(fabsf(lat[r]), v[r], acc);
    } else {
#pragma unroll
      for (int r = 0; r < 64; ++r) acc = fmaf(lat[r], v[r], acc);
    }
  } else if ((p.rank & 7) == 0) {
    for (int r = 0; r < p.rank; r += 8) {
      float v[8];
      Vec8<WT>::load(row + r, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(p.legacy ? fabsf(lat[r + e]) : lat[r + e], v[e], acc);
    }
  } else {
    for (int r = 0; r < p.rank; ++r) acc = fmaf(p.legacy ? fabsf(lat[r]) : lat[r], to_f32(row[r]), acc);
  }
  if (!p.legacy) {
    if (p.score_b != nullptr) acc += to_f32(reinterpret_cast<const WT*>(p.score_b)[b]);
    acc = fmaxf(acc, 0.f);
  }
  if (p.dbn != nullptr) acc *= p.dbn[b];
  return acc;
}

// The router kernel's partial latents reduced in fixed order -- every scores
// CTA computes the same values, then the RMSNorm scale, enc_b and the basis
// top-k mask apply (streaming_llama_runtime.py:4220-4238).  Rank 64 with a
// multiple of 8 partials (the decode shapes): thread (column quad c4, group g)
// sums partials g, g+8, ... with all of its 16-byte loads in flight, and the 8
// group sums combine in order; other shapes: thread (row r, half h) sums
// partials h, h+2, ... and the halves combine.
__device__ __forceinline__ void reduce_latent(const RouterBParams& p, float* lat, float enc_b_own = 0.f) {
  __shared__ float grp[8][kMaxRank];
  __shared__ float s_norm;
  const int tid = threadIdx.x, lane = tid & 31;
  const float* lpart = p.ws.latent_part + (int64_t)blockIdx.y * kRouterMaxCtas * p.rank;  // row blockIdx.y
  if (tid < 32) {
    const float* sp = p.ws.sumsq_part + blockIdx.y * kRouterMaxCtas;
    float v[kRouterMaxCtas / 32];
#pragma unroll
    for (int u = 0; u < kRouterMaxCtas / 32; ++u) {
      const int b = lane + 32 * u;
      v[u] = (p.use_norm && b < p.nparts) ? ldcg_f32(sp + b) : 0.f;
    }
    float t = 0.f;
#pragma unroll
    for (int u = 0; u < kRouterMaxCtas / 32; ++u) t += v[u];
    t = warp_sum(t);
    if (lane == 0) s_norm = p.use_norm ? 1.f / sqrtf(t / (float)p.H + p.eps) : 1.f;
  }
  int ngroups;
  if (p.rank == 64 && (p.nparts & 7) == 0 && p.nparts <= 128 && blockDim.x == 128) {
    ngroups = 8;
    const int c4 = tid & 15, g = tid >> 4;
    const float4* base = reinterpret_cast<const float4*>(lpart) + c4;
    float4 v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int b = g + 8 * u;
      v[u] = b < p.nparts ? __ldcg(base + b * 16) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      a.x += v[u].x;
      a.y += v[u].y;
      a.z += v[u].z;
      a.w += v[u].w;
    }
    grp[g][4 * c4 + 0] = a.x;
    grp[g][4 * c4 + 1] = a.y;
    grp[g][4 * c4 + 2] = a.z;
    grp[g][4 * c4 + 3] = a.w;
  } else {
    ngroups = 2;
    for (int e = tid; e < 2 * p.rank; e += blockDim.x) {
      const int r = e % p.rank, h = e / p.rank;
      float acc = 0.f;
      int b = h;
      for (; b + 14 < p.nparts; b += 16) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = ldcg_f32(&lpart[(b + 2 * u) * p.rank + r]);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc += v[u];
      }
      for (; b < p.nparts; b += 2) acc += ldcg_f32(&lpart[b * p.rank + r]);
      grp[h][r] = acc;
    }
  }
  __syncthreads();
  for (int r = tid; r < p.rank; r += blockDim.x) {
    float acc = 0.f;
    for (int g = 0; g < ngroups; ++g) acc += grp[g][r];
    acc *= s_norm;
    // enc_b_own: enc_b[tid], loaded by the caller before its upstream wait
    if (p.enc_b != nullptr) acc += r == tid ? enc_b_own : load_as_f32(p.enc_b, p.wdtype, r);
    lat[r] = acc;
  }
  __syncthreads();
  const int bk = max(1, min(p.basis_top_k, p.rank));
  if (bk < p.rank) {
    float keep[2] = {0.f, 0.f};
    for (int r = tid, j = 0; r < p.rank; r += blockDim.x, ++j) {
      const float a = fabsf(lat[r]);
      int pos = 0;
      for (int q = 0; q < p.rank; ++q) {
        const float b = fabsf(lat[q]);
        pos += (b > a) || (b == a && q < r);
      }
      keep[j] = pos < bk ? lat[r] : 0.f;
    }
    __syncthreads();
    for (int r = tid, j = 0; r < p.rank; r += blockDim.x, ++j) lat[r] = keep[j];
    __syncthreads();
  }
  if (blockIdx.x == 0) {
    for (int r = tid; r < p.rank; r += blockDim.x) p.ws.latent[blockIdx.y * p.rank + r] = lat[r];
    if (tid == 0 && !p.multi_rows) {
      *p.ws.norm_scale = s_norm;
      if (p.epoch_counter) *p.epoch_counter = *p.epoch_counter + 1u;  // this rank finished its exchange
    }
  }
}

// Block scores, one thread per block (grid-wide; waits for the latent).  At
// rank 64 with 2-byte weights the thread's score-head row is loaded before the
// wait on the upstream kernels (weights are not written upstream).
template <typename WT>
__global__ void __launch_bounds__(128) router_scores_kernel(RouterBParams p) {
  __shared__ float lat[kMaxRank];
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  const bool pre = sizeof(WT) == 2 && p.rank == 64 && b < p.NB;
  uint4 wrow[8];
  float sbias = 0.f, dbn = 1.f;
  if (pre) {
    const uint4* row = reinterpret_cast<const uint4*>(reinterpret_cast<const WT*>(p.score_w) + (int64_t)b * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) wrow[i] = __ldg(row + i);
    if (p.score_b != nullptr) sbias = to_f32(reinterpret_cast<const WT*>(p.score_b)[b]);
    if (p.dbn != nullptr) dbn = p.dbn[b];
  }
  const float enc_b_own =
      (p.reduce_latent && p.enc_b != nullptr && (int)threadIdx.x < p.rank) ? load_as_f32(p.enc_b, p.wdtype, threadIdx.x)
                                                                           : 0.f;
  pdl_trigger();
  pdl_wait();
  if (p.reduce_latent) {
    reduce_latent(p, lat, enc_b_own);
  } else {
    for (int r = threadIdx.x; r < p.rank; r += blockDim.x) lat[r] = ldcg_f32(&p.ws.latent[r + blockIdx.y * p.rank]);
    __syncthreads();
  }
  if (pre) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t w4[4] = {wrow[i].x, wrow[i].y, wrow[i].z, wrow[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float lo, hi;
        if (std::is_same<WT, __half>::value) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[e]));
          lo = f.x;
          hi = f.y;
        } else {
          lo = __uint_as_float(w4[e] << 16);
          hi = __uint_as_float(w4[e] & 0xffff0000u);
        }
        const int r = i * 8 + 2 * e;
        acc = fmaf(p.legacy ? fabsf(lat[r]) : lat[r], lo, acc);
        acc = fmaf(p.legacy ? fabsf(lat[r + 1]) : lat[r + 1], hi, acc);
      }
    }
    if (!p.legacy) {
      if (p.score_b != nullptr) acc += sbias;
      acc = fmaxf(acc, 0.f);
    }
    if (p.dbn != nullptr) acc *= dbn;
    p.ws.scores[(int64_t)blockIdx.y * p.NB + b] = acc;
    return;
  }
  if (b < p.NB) p.ws.scores[(int64_t)blockIdx.y * p.NB + b] = score_row<WT>(p, lat, b);
}

// Top-k of the block scores in one CTA of 1024 threads: radix select of the
// k-th largest order-preserving key (8-bit digits, warp-aggregated histogram
// increments), threshold ties resolved by lower block id.  The winners are
// compacted in block-id order; when the caller wants the indices they are
// also ordered score-descending (ties: lower id first) by a bitonic sort.
__global__ void __launch_bounds__(1024) router_topk_kernel(RouterBParams p) {
  extern __shared__ uint32_t keys[];  // [NB]
  __shared__ RadixSelectSmem S;
  __shared__ unsigned long long sorted[1024];
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x;
  const int NB = p.NB, k = p.top_k;
  const bool want_order = p.idx_out != nullptr || p.score_out != nullptr;
  const int row = p.multi_rows ? blockIdx.x : 0;
  int32_t* idx_out = p.idx_out ? p.idx_out + (int64_t)row * k : nullptr;
  float* score_out = p.score_out ? p.score_out + (int64_t)row * k : nullptr;
  int* sel_idx = p.ws.sel_idx + (int64_t)row * k;
  // the keys' common leading bits need no pass: digits start below them
  uint32_t kor = 0u, kand = 0xffffffffu;
  {
    constexpr int kPer = kMaxNumBlocks / 1024;  // all of this thread's score loads in flight
    float v[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = u * (int)blockDim.x + tid;
      v[u] = i < NB ? ldcg_f32(&p.ws.scores[(int64_t)row * NB + i]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = u * (int)blockDim.x + tid;
      if (i < NB) {
        const uint32_t key = orderable(v[u]);
        keys[i] = key;
        kor |= key;
        kand &= key;
      }
    }
  }
  block_radix_select(keys, NB, k, kor, kand, S);
  const uint32_t thr = S.prefix;
  const int take_eq = S.need;
  // winners in block-id order (contiguous chunk per thread)
  const int per = (NB + blockDim.x - 1) / blockDim.x;
  const int lo = min(NB, tid * per), hi = min(NB, lo + per);
  const bool ordered = want_order;
  if (!ordered && take_eq == S.bin_count) {
    // no tie is split at the threshold: the selection is key >= thr; one scan
    // compacts the selected blocks present here into pool rows (block-id order)
    int m = 0;
    for (int i = lo; i < hi; ++i) m += keys[i] >= thr && map_block(p, i) >= 0;
    int tot;
    int pos = block_exclusive_scan(m, &tot);
    for (int i = lo; i < hi; ++i) {
      if (keys[i] < thr) continue;
      const int r = map_block(p, i);
      if (r < 0) continue;
      p.ws.rows[pos] = r;
      p.ws.row_block[pos] = i;
      ++pos;
    }
    if (p.latent_out)
      for (int r = tid; r < p.rank; r += blockDim.x) p.latent_out[r] = ldcg_f32(&p.ws.latent[r]);
    if (tid == 0) *p.ws.count = tot;
    return;
  }
  int n_eq = 0, n_gt = 0;
  for (int i = lo; i < hi; ++i) {
    n_eq += keys[i] == thr;
    n_gt += keys[i] > thr;
  }
  int tot;
  const int eq_before = block_exclusive_scan(n_eq, &tot);
  const int my_sel = n_gt + max(0, min(n_eq, take_eq - eq_before));
  const int sel_before = block_exclusive_scan(my_sel, &tot);
  {
    int e = eq_before, out = sel_before;
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = keys[i];
      bool s = key > thr;
      if (key == thr) {
        s = e < take_eq;
        ++e;
      }
      if (s) {
        sel_idx[out] = i;
        if (ordered && out < 1024) sorted[out] = ((unsigned long long)key << 32) | (0xffffffffu - (uint32_t)i);
        ++out;
      }
    }
  }
  if (p.latent_out)
    for (int r = tid; r < p.rank; r += blockDim.x)
      p.latent_out[(int64_t)row * p.rank + r] = ldcg_f32(&p.ws.latent[(int64_t)row * p.rank + r]);
  __threadfence_block();
  __syncthreads();
  if (ordered) {
    if (k <= 1024) {
      int n2 = 1;
      while (n2 < k) n2 <<= 1;
      for (int i = k + tid; i < n2; i += blockDim.x) sorted[i] = 0ull;
      __syncthreads();
      for (int len = 2; len <= n2; len <<= 1) {
        for (int j = len >> 1; j > 0; j >>= 1) {
          for (int i = tid; i < n2; i += blockDim.x) {
            const int ixj = i ^ j;
            if (ixj > i) {
              const unsigned long long a = sorted[i], b = sorted[ixj];
              const bool desc = (i & len) == 0;
              if (desc ? (a < b) : (a > b)) {
                sorted[i] = b;
                sorted[ixj] = a;
              }
            }
          }
          __syncthreads();
        }
      }
      for (int j = tid; j < k; j += blockDim.x) {
        const unsigned long long key = sorted[j];
        const int id = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
        if (idx_out) idx_out[j] = id;
        if (score_out) score_out[j] = from_orderable((uint32_t)(key >> 32));
      }
    } else {
      // large k: rank of every block among all blocks (exact, slower)
      for (int i = tid; i < NB; i += blockDim.x) {
        const uint32_t ki = keys[i];
        int pos = 0;
        for (int q = 0; q < NB; ++q) {
          const uint32_t kq = keys[q];
          pos += (kq > ki) || (kq == ki && q < i);
        }
        if (pos < k) {
          if (idx_out) idx_out[pos] = i;
          if (score_out) score_out[pos] = from_orderable(ki);
        }
      }
    }
  }
  if (p.multi_rows) return;  // routing only: no pool rows
  compact_selection(p, sel_idx, k);
}

__global__ void __launch_bounds__(512) select_given_kernel(RouterBParams p, const int32_t* idx_in, int k) {
  pdl_trigger();
  pdl_wait();
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int b = idx_in[j];
    p.ws.sel_idx[j] = (b >= 0 && b < p.NB) ? b : -1;
  }
  __syncthreads();
  compact_selection(p, p.ws.sel_idx, k);
}

// ---------------------------------------------------------------------------
// launches
// ---------------------------------------------------------------------------
int router_setup() {
  static bool done[64] = {};
  int dev = 0;
  NSM_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && done[dev]) return NSM_OK;
  NSM_CHECK_CUDA(
      cudaFuncSetAttribute(router_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxNumBlocks * 4));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return NSM_OK;
}

int router_a_ctas(int H, int* cols_per_cta) {
  int ctas = std::max(1, (H + 127) / 128);
  int cpc = 128;
  if (ctas > kRouterMaxCtas) {
    cpc = ((H + kRouterMaxCtas - 1) / kRouterMaxCtas + 63) / 64 * 64;
    ctas = (H + cpc - 1) / cpc;
  }
  *cols_per_cta = cpc;
  return ctas;
}

int router_a_launch(const RouterAParams& a_in, cudaStream_t stream) {
  RouterAParams a = a_in;
  int cpc;
  const int ctas = router_a_ctas(a.H, &cpc);
  a.cols_per_cta = cpc;
  const size_t smem = 2 * (size_t)cpc * sizeof(float);
  cudaError_t e;
  switch (a.wdtype) {
    case NSM_F32: e = launch_pdl(router_latent_kernel<float>, ctas, 256, smem, stream, a); break;
    case NSM_F16: e = launch_pdl(router_latent_kernel<__half>, ctas, 256, smem, stream, a); break;
    default: e = launch_pdl(router_latent_kernel<__nv_bfloat16>, ctas, 256, smem, stream, a); break;
  }
  NSM_CHECK_CUDA(e);
  return NSM_OK;
}

int router_b_launch(const RouterBParams& b, cudaStream_t stream, bool topk) {
  int st = router_setup();
  if (st) return st;
  const int ctas = (b.NB + 127) / 128;
  cudaError_t e;
  switch (b.wdtype) {
    case NSM_F32: e = launch_pdl(router_scores_kernel<float>, ctas, 128, 0, stream, b); break;
    case NSM_F16: e = launch_pdl(router_scores_kernel<__half>, ctas, 128, 0, stream, b); break;
    default: e = launch_pdl(router_scores_kernel<__nv_bfloat16>, ctas, 128, 0, stream, b); break;
  }
  NSM_CHECK_CUDA(e);
  if (topk) NSM_CHECK_CUDA(launch_pdl(router_topk_kernel, 1, 1024, (size_t)b.NB * 4, stream, b));
  return NSM_OK;
}

int router_rows_launch(const RouterAParams& a_in, RouterBParams b, int rows, cudaStream_t stream) {
  int st = router_setup();
  if (st) return st;
  RouterAParams a = a_in;
  int cpc;
  const int ctas = router_a_ctas(a.H, &cpc);
  a.cols_per_cta = cpc;
  a.reduce_in_scores = 1;
  a.multi_rows = rows;
  b.multi_rows = rows;
  b.reduce_latent = 1;
  b.nparts = ctas;
  b.use_norm = 0;
  b.H = a.H;
  b.enc_b = a.enc_b;
  b.basis_top_k = a.basis_top_k;
  const size_t smem = (size_t)std::min(rows, kLatentRowsPerCta) * cpc * sizeof(float);
  const dim3 ga(ctas, (rows + kLatentRowsPerCta - 1) / kLatentRowsPerCta), gb((b.NB + 127) / 128, rows);
  cudaError_t e;
  switch (a.wdtype) {
    case NSM_F32: e = launch_pdl(router_latent_kernel<float>, ga, 256, smem, stream, a); break;
    case NSM_F16: e = launch_pdl(router_latent_kernel<__half>, ga, 256, smem, stream, a); break;
    default: e = launch_pdl(router_latent_kernel<__nv_bfloat16>, ga, 256, smem, stream, a); break;
  }
  NSM_CHECK_CUDA(e);
  switch (b.wdtype) {
    case NSM_F32: e = launch_pdl(router_scores_kernel<float>, gb, 128, 0, stream, b); break;
    case NSM_F16: e = launch_pdl(router_scores_kernel<__half>, gb, 128, 0, stream, b); break;
    default: e = launch_pdl(router_scores_kernel<__nv_bfloat16>, gb, 128, 0, stream, b); break;
  }
  NSM_CHECK_CUDA(e);
  NSM_CHECK_CUDA(launch_pdl(router_topk_kernel, rows, 1024, (size_t)b.NB * 4, stream, b));
  return NSM_OK;
}

int select_given_launch(const RouterBParams& b, const int32_t* idx_in, int k, cudaStream_t stream) {
  NSM_CHECK_CUDA(launch_pdl(select_given_kernel, 1, 512, 0, stream, b, idx_in, k));
  return NSM_OK;
}

}  // namespace nsm
