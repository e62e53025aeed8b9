// nsm_decode.cu -- single-token blockwise-sparse NF4 decode MLP for sm_100a.
//
// Pipeline of one decode step (one decoder layer, one token), all on one stream:
//   1. router_latent_kernel   x prep (optional residual add + RMSNorm), fp16 x
//                             with per-64-column power-of-two scales, split-H
//                             partial latent x . enc_w^T; the last CTA reduces,
//                             applies the norm scale, bias and basis top-k.
//   2. router_select_kernel   block scores clamp0(latent . score_w^T + b)
//                             (* down_block_norm), the last CTA sorts (score
//                             desc, index asc), emits the top-k and compacts
//                             the selection into pool rows through the block
//                             map (resident table or shard range).
//   3. gateup_kernel          persistent warps over (block, column-range)
//                             units: NF4 gather-GEMV of gate and up, fp32
//                             partials, the last unit of a block reduces them
//                             in fixed order and writes SiLU(g)*u as fp16 with
//                             a per-block power-of-two scale.
//   4. down_kernel            persistent warps over (32-row tile, block group)
//                             units: NF4 column gather-GEMV, split-K partials,
//                             the last group of a row tile reduces in fixed
//                             order and writes y.
// Reference semantics: streaming_llama_runtime.py:4209-4238 (latent),
// :4311-4352 (scores/top-k), :5433-5492 (MLP math).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <string>

#include "nsm_common.cuh"
#include "nsm_internal.h"

namespace nsm {

// ============================================================================
// 1. router latent (+ x preparation)
// ============================================================================
struct RouterAParams {
  const void* x;
  int x_dtype;
  float* residual;
  const void* y_prev;
  int y_prev_dtype;
  const void* norm_w;
  int norm_w_dtype;
  float eps;
  int use_norm;
  const void* enc_w;  // may be null: x preparation only
  const void* enc_b;
  int wdtype;
  int rank;
  int basis_top_k;
  int H;
  int cols_per_cta;  // multiple of 64
  DecodeWs ws;
};

__global__ void __launch_bounds__(256) router_latent_kernel(RouterAParams p) {
  extern __shared__ float xs[];  // [cols_per_cta]
  __shared__ float red[32];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c0 = blockIdx.x * p.cols_per_cta;
  const int c1 = min(p.H, c0 + p.cols_per_cta);
  const int n = c1 - c0;

  float sumsq = 0.f;
  for (int i = tid; i < n; i += blockDim.x) {
    const int c = c0 + i;
    float v;
    if (p.residual != nullptr) {
      v = p.residual[c];
      if (p.y_prev != nullptr) v += load_as_f32(p.y_prev, p.y_prev_dtype, c);
      p.residual[c] = v;
      sumsq += v * v;
      if (p.norm_w != nullptr) v *= load_as_f32(p.norm_w, p.norm_w_dtype, c);
    } else {
      v = load_as_f32(p.x, p.x_dtype, c);
    }
    xs[i] = v;
  }
  sumsq = warp_sum(sumsq);
  if (lane == 0) red[warp] = sumsq;
  __syncthreads();
  if (tid == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    p.ws.sumsq_part[blockIdx.x] = t;
  }

  // fp16 copy of x with a power-of-two scale per 64-column tile
  const int ntiles = n >> 6;
  for (int tl = warp; tl < ntiles; tl += (blockDim.x >> 5)) {
    const float a = xs[tl * 64 + lane], b = xs[tl * 64 + 32 + lane];
    const float m = warp_max(fmaxf(fabsf(a), fabsf(b)));
    const float s = pow2_scale_for(m);
    const float inv = 1.f / s;  // exact: s is a power of two
    const int c = c0 + tl * 64;
    p.ws.x16[c + lane] = __float2half_rn(a * inv);
    p.ws.x16[c + 32 + lane] = __float2half_rn(b * inv);
    if (lane == 0) p.ws.xscale[c >> 6] = s;
  }

  if (p.enc_w != nullptr) {
    for (int r = warp; r < p.rank; r += (blockDim.x >> 5)) {
      float acc = 0.f;
      const int64_t rowoff = (int64_t)r * p.H + c0;
      for (int i = lane; i < n; i += 32) acc += load_as_f32(p.enc_w, p.wdtype, rowoff + i) * xs[i];
      acc = warp_sum(acc);
      if (lane == 0) p.ws.latent_part[blockIdx.x * p.rank + r] = acc;
    }
  }

  // last CTA: reduce partials in CTA order
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(p.ws.ticket_router_a, 1);
    s_last = (prev == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  __shared__ float s_norm;
  __shared__ float lat[kMaxRank];
  if (tid == 0) {
    float ns = 1.f;
    if (p.use_norm) {
      double t = 0.0;
      for (int b = 0; b < (int)gridDim.x; ++b) t += (double)ldcg_f32(&p.ws.sumsq_part[b]);
      const float var = (float)(t / (double)p.H);
      ns = 1.f / sqrtf(var + p.eps);
    }
    s_norm = ns;
    *p.ws.norm_scale = ns;
  }
  __syncthreads();
  if (p.enc_w != nullptr) {
    for (int r = tid; r < p.rank; r += blockDim.x) {
      float acc = 0.f;
      for (int b = 0; b < (int)gridDim.x; ++b) acc += ldcg_f32(&p.ws.latent_part[b * p.rank + r]);
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
        int rank_pos = 0;
        for (int q = 0; q < p.rank; ++q) {
          const float b = fabsf(lat[q]);
          rank_pos += (b > a) || (b == a && q < r);
        }
        if (rank_pos >= bk) v = 0.f;
      }
      p.ws.latent[r] = v;
    }
  }
  if (tid == 0) *p.ws.ticket_router_a = 0;
}

// ============================================================================
// 2. block scores + top-k + selection -> pool rows
// ============================================================================
struct RouterBParams {
  const void* score_w;
  const void* score_b;
  int wdtype;
  const float* dbn;
  int legacy;
  int rank;
  int NB;
  int top_k;
  int sort_n;  // power of two >= NB
  int32_t* idx_out;
  float* score_out;
  float* latent_out;
  const int32_t* slot_of_block;
  int block_begin;
  int block_end;
  int pool_rows;
  DecodeWs ws;
};

__device__ __forceinline__ uint32_t orderable(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_orderable(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

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

// exclusive block scan of 0/1 flags, writes compacted pool rows
__device__ void compact_selection(const RouterBParams& p, const int* sel, int k) {
  __shared__ int warp_tot[32];
  __shared__ int s_base;
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int j0 = 0; j0 < k; j0 += blockDim.x) {
    const int j = j0 + threadIdx.x;
    int r = -1;
    if (j < k) r = map_block(p, sel[j]);
    const int f = r >= 0;
    const unsigned bal = __ballot_sync(0xffffffffu, f);
    const int pre = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += warp_tot[w];
    if (f) {
      p.ws.rows[s_base + wbase + pre] = r;
      p.ws.row_block[s_base + wbase + pre] = sel[j];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int w = 0; w < nw; ++w) t += warp_tot[w];
      s_base += t;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *p.ws.count = s_base;
}

__global__ void __launch_bounds__(512) router_select_kernel(RouterBParams p) {
  extern __shared__ unsigned long long keys[];  // [sort_n] (last CTA only)
  __shared__ float lat[kMaxRank];
  __shared__ int s_last;
  const int tid = threadIdx.x;
  for (int r = tid; r < p.rank; r += blockDim.x) lat[r] = ldcg_f32(&p.ws.latent[r]);
  __syncthreads();
  for (int b = blockIdx.x * blockDim.x + tid; b < p.NB; b += gridDim.x * blockDim.x) {
    float acc = 0.f;
    const int64_t off = (int64_t)b * p.rank;
    if (p.legacy) {
      for (int r = 0; r < p.rank; ++r) acc += fabsf(lat[r]) * load_as_f32(p.score_w, p.wdtype, off + r);
    } else {
      for (int r = 0; r < p.rank; ++r) acc += lat[r] * load_as_f32(p.score_w, p.wdtype, off + r);
      if (p.score_b != nullptr) acc += load_as_f32(p.score_b, p.wdtype, b);
      acc = fmaxf(acc, 0.f);
    }
    if (p.dbn != nullptr) acc *= p.dbn[b];
    p.ws.scores[b] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(p.ws.ticket_router_b, 1);
    s_last = (prev == (int)gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = tid; i < p.sort_n; i += blockDim.x) {
    unsigned long long key = 0ull;
    if (i < p.NB) {
      const float s = ldcg_f32(&p.ws.scores[i]);
      key = ((unsigned long long)orderable(s) << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
    }
    keys[i] = key;
  }
  __syncthreads();
  // bitonic sort, descending
  for (int k = 2; k <= p.sort_n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < p.sort_n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = keys[i], b = keys[ixj];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const int k = p.top_k;
  for (int j = tid; j < k; j += blockDim.x) {
    const unsigned long long key = keys[j];
    const int idx = (int)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    p.ws.sel_idx[j] = idx;
    if (p.idx_out) p.idx_out[j] = idx;
    if (p.score_out) p.score_out[j] = from_orderable((uint32_t)(key >> 32));
  }
  if (p.latent_out) {
    for (int r = tid; r < p.rank; r += blockDim.x) p.latent_out[r] = lat[r];
  }
  __syncthreads();
  compact_selection(p, p.ws.sel_idx, k);
  if (tid == 0) *p.ws.ticket_router_b = 0;
}

// Selection supplied by the caller: copy + compaction (single CTA).
__global__ void __launch_bounds__(512) select_given_kernel(RouterBParams p, const int32_t* idx_in, int k) {
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    const int b = idx_in[j];
    p.ws.sel_idx[j] = (b >= 0 && b < p.NB) ? b : -1;
  }
  __syncthreads();
  // invalid ids map to "not present"
  compact_selection(p, p.ws.sel_idx, k);
}

// Identity rows 0..count-1 (gathered layouts).
__global__ void identity_rows_kernel(int* rows, int* count, int* sel, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    rows[i] = i;
    sel[i] = i;
  }
  // (row i of a gathered layout is block i of the gathered list)
  if (blockIdx.x == 0 && threadIdx.x == 0) *count = n;
}

// ============================================================================
// 3. gate/up gather-GEMV + SiLU*up
// ============================================================================
struct GateUpParams {
  const uint8_t* gate;
  const float* gate_am;
  const uint8_t* up;
  const float* up_am;
  int64_t gstride;   // bytes between pool rows (blocks)
  int64_t gastride;  // floats between pool rows
  const float* gate_code;
  const float* up_code;
  const void* gate_bias;
  const void* up_bias;
  int bias_dtype;
  int bias_by_block;  // 1: bias index = row_block[s]*32+l, 0: s*32+l
  int H;
  const int* rows;
  const int* count_ptr;
  const int* row_block;  // block id of compacted slot s
  const __half* x16;
  const float* xscale;
  const float* norm_scale;
  const void* act_mask;  // optional [U*32] (one row of flat_mask)
  int mask_dtype;
  float* gu_part;
  int* ticket_slot;
  __half* act16;
  float* act_scale;
  float* act_out;  // optional fp32 [k][32]
  int total_warps;
};

struct TileRegs {
  uint2 w[2][2][2];  // [proj][rowgroup][row g / g+8]
  float am[2][2][2];
};

__device__ __forceinline__ void gateup_load_tile(const GateUpParams& p, const uint8_t* gbase, const uint8_t* ubase,
                                                 const float* gab, const float* uab, int j, int g, int t,
                                                 TileRegs& r) {
  const int bpr = p.H >> 1;   // bytes per row
  const int apr = p.H >> 6;   // absmax per row
#pragma unroll
  for (int rg = 0; rg < 2; ++rg) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = rg * 16 + g + h * 8;
      const int64_t boff = (int64_t)row * bpr + j * 32 + t * 8;
      r.w[0][rg][h] = ldg_stream_u2(gbase + boff);
      r.w[1][rg][h] = ldg_stream_u2(ubase + boff);
      r.am[0][rg][h] = ldg_f32(gab + (int64_t)row * apr + j);
      r.am[1][rg][h] = ldg_f32(uab + (int64_t)row * apr + j);
    }
  }
}

template <int kTable>
__device__ __forceinline__ void gateup_mma_rowgroup(const uint32_t* lut, uint32_t lanebase, const uint2 w0,
                                                    const uint2 w1, const uint32_t b[8], float d[4]) {
  d[0] = d[1] = d[2] = d[3] = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t x0 = c < 2 ? w0.x : w0.y;
    const uint32_t x1 = c < 2 ? w1.x : w1.y;
    const int kb = (c & 1) * 2;
    const uint32_t a0 = lut_lookup_rt(lut, x0, lanebase, kb, kTable);
    const uint32_t a1 = lut_lookup_rt(lut, x1, lanebase, kb, kTable);
    const uint32_t a2 = lut_lookup_rt(lut, x0, lanebase, kb + 1, kTable);
    const uint32_t a3 = lut_lookup_rt(lut, x1, lanebase, kb + 1, kTable);
    mma_16816(d, a0, a1, a2, a3, b[2 * c], b[2 * c + 1]);
  }
}

__device__ __forceinline__ int gateup_tiles_per_unit(int count, int tiles_per_row, int total_warps) {
  const int min_tpu = (tiles_per_row + kMaxUnitsPerSlot - 1) / kMaxUnitsPerSlot;
  const long long total = (long long)count * tiles_per_row;
  long long want = total / (4LL * total_warps);
  int tpu = (int)max(1LL, min(16LL, want));
  return max(tpu, min_tpu);
}

__global__ void __launch_bounds__(256, 2) gateup_kernel(GateUpParams p) {
  extern __shared__ __align__(16) uint32_t lut[];
  build_lut(lut, p.gate_code, p.up_code);
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lanebase = (uint32_t)lane * 4u;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int count = *p.count_ptr;
  const int tiles_per_row = p.H >> 6;
  const int tpu = gateup_tiles_per_unit(count, tiles_per_row, p.total_warps);
  const int ups = (tiles_per_row + tpu - 1) / tpu;
  const int nunits = count * ups;

  for (int u = warp_global; u < nunits; u += p.total_warps) {
    const int s = u / ups, sub = u - s * ups;
    const int prow = p.rows[s];
    const uint8_t* gbase = p.gate + (int64_t)prow * p.gstride;
    const uint8_t* ubase = p.up + (int64_t)prow * p.gstride;
    const float* gab = p.gate_am + (int64_t)prow * p.gastride;
    const float* uab = p.up_am + (int64_t)prow * p.gastride;
    const int j0 = sub * tpu, j1 = min(tiles_per_row, j0 + tpu);
    float acc[2][2][2] = {};  // [proj][rg][h]
    TileRegs cur, nxt;
    gateup_load_tile(p, gbase, ubase, gab, uab, j0, g, t, cur);
    for (int j = j0; j < j1; ++j) {
      if (j + 1 < j1) gateup_load_tile(p, gbase, ubase, gab, uab, j + 1, g, t, nxt);
      uint32_t b[8];
      {
        const uint4 xa = ldg_u4(p.x16 + j * 64 + t * 16);
        const uint4 xb = ldg_u4(p.x16 + j * 64 + t * 16 + 8);
        b[0] = xa.x; b[1] = xa.y; b[2] = xa.z; b[3] = xa.w;
        b[4] = xb.x; b[5] = xb.y; b[6] = xb.z; b[7] = xb.w;
      }
      const float xs = ldg_f32(p.xscale + j);
#pragma unroll
      for (int rg = 0; rg < 2; ++rg) {
        float d[4];
        gateup_mma_rowgroup<0>(lut, lanebase, cur.w[0][rg][0], cur.w[0][rg][1], b, d);
        acc[0][rg][0] = fmaf(d[0], cur.am[0][rg][0] * xs, acc[0][rg][0]);
        acc[0][rg][1] = fmaf(d[2], cur.am[0][rg][1] * xs, acc[0][rg][1]);
        gateup_mma_rowgroup<1>(lut, lanebase, cur.w[1][rg][0], cur.w[1][rg][1], b, d);
        acc[1][rg][0] = fmaf(d[0], cur.am[1][rg][0] * xs, acc[1][rg][0]);
        acc[1][rg][1] = fmaf(d[2], cur.am[1][rg][1] * xs, acc[1][rg][1]);
      }
      cur = nxt;
    }
    // column 0 of the accumulator lives in lanes with t == 0
    float* part = p.gu_part + ((int64_t)s * kMaxUnitsPerSlot + sub) * 64;
    if (t == 0) {
#pragma unroll
      for (int pr = 0; pr < 2; ++pr)
#pragma unroll
        for (int rg = 0; rg < 2; ++rg)
#pragma unroll
          for (int h = 0; h < 2; ++h) part[pr * 32 + rg * 16 + g + h * 8] = acc[pr][rg][h];
      __threadfence();
    }
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      const int prev = atomicAdd(&p.ticket_slot[s], 1);
      last = prev == ups - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    float gsum = 0.f, usum = 0.f;
    const float* base = p.gu_part + (int64_t)s * kMaxUnitsPerSlot * 64;
    for (int q = 0; q < ups; ++q) {
      gsum += ldcg_f32(base + q * 64 + lane);
      usum += ldcg_f32(base + q * 64 + 32 + lane);
    }
    const float ns = p.norm_scale ? ldcg_f32(p.norm_scale) : 1.f;
    gsum *= ns;
    usum *= ns;
    if (p.gate_bias != nullptr || p.up_bias != nullptr) {
      const int bi = (p.bias_by_block ? p.row_block[s] : s) * 32 + lane;
      if (p.gate_bias) gsum += load_as_f32(p.gate_bias, p.bias_dtype, bi);
      if (p.up_bias) usum += load_as_f32(p.up_bias, p.bias_dtype, bi);
    }
    if (p.act_mask != nullptr) {
      const float m = load_as_f32(p.act_mask, p.mask_dtype, (int64_t)s * 32 + lane);
      gsum *= m;
      usum *= m;
    }
    const float act = silu_f32(gsum) * usum;
    if (p.act_out) p.act_out[(int64_t)s * 32 + lane] = act;
    const float m = warp_max(fabsf(act));
    const float sc = pow2_scale_for(m);
    p.act16[(int64_t)s * 32 + lane] = __float2half_rn(act * (1.f / sc));
    if (lane == 0) {
      p.act_scale[s] = sc;
      p.ticket_slot[s] = 0;
    }
  }
}

// ============================================================================
// 4. down column gather-GEMV (split-K over blocks)
// ============================================================================
struct DownParams {
  const uint8_t* down;
  const float* down_am;
  int64_t dbs, drs, dabs, dars;
  int pair;
  const float* down_code;
  const void* down_bias;
  int bias_dtype;
  int H;
  const int* rows;
  const int* count_ptr;
  const __half* act16;
  const float* act_scale;
  float* ypart;
  int* ticket_rt;
  void* y;
  int y_dtype;
  int total_warps;
};

__global__ void __launch_bounds__(256, 2) down_kernel(DownParams p) {
  extern __shared__ __align__(16) uint32_t lut[];
  build_lut(lut, p.down_code, p.down_code);
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t lanebase = (uint32_t)lane * 4u;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int count = *p.count_ptr;
  const int RT = p.H >> 5;
  int sg = (4 * p.total_warps + RT - 1) / RT;
  sg = max(1, min(sg, min(max(count, 1), kMaxSlotGroups)));
  const int gs = (count + sg - 1) / sg;
  const int nunits = RT * sg;

  for (int u = warp_global; u < nunits; u += p.total_warps) {
    const int grp = u / RT, rt = u - grp * RT;
    const int s0 = grp * gs, s1 = min(count, s0 + gs);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8, 16+g, 24+g
    for (int s = s0; s < s1; ++s) {
      const int prow = p.rows[s];
      const uint8_t* base = p.down + (int64_t)prow * p.dbs;
      const float* abase = p.down_am + (int64_t)(p.pair ? (prow >> 1) : prow) * p.dabs;
      uint32_t w[4];
      float am[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = rt * 32 + (i >> 1) * 16 + g + (i & 1) * 8;
        w[i] = ldg_u32(base + (int64_t)row * p.drs + t * 4);
        am[i] = ldg_f32(abase + (int64_t)row * p.dars);
      }
      const uint4 bf = ldg_u4(p.act16 + (int64_t)s * 32 + t * 8);
      const float as = ldg_f32(p.act_scale + s);
      const uint32_t b[4] = {bf.x, bf.y, bf.z, bf.w};
#pragma unroll
      for (int rg = 0; rg < 2; ++rg) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint32_t a0 = lut_lookup_rt(lut, w[rg * 2], lanebase, 2 * c, 0);
          const uint32_t a1 = lut_lookup_rt(lut, w[rg * 2 + 1], lanebase, 2 * c, 0);
          const uint32_t a2 = lut_lookup_rt(lut, w[rg * 2], lanebase, 2 * c + 1, 0);
          const uint32_t a3 = lut_lookup_rt(lut, w[rg * 2 + 1], lanebase, 2 * c + 1, 0);
          mma_16816(d, a0, a1, a2, a3, b[2 * c], b[2 * c + 1]);
        }
        acc[rg * 2] = fmaf(d[0], am[rg * 2] * as, acc[rg * 2]);
        acc[rg * 2 + 1] = fmaf(d[2], am[rg * 2 + 1] * as, acc[rg * 2 + 1]);
      }
    }
    if (t == 0) {
      float* yp = p.ypart + (int64_t)grp * p.H + rt * 32;
#pragma unroll
      for (int i = 0; i < 4; ++i) yp[(i >> 1) * 16 + g + (i & 1) * 8] = acc[i];
      __threadfence();
    }
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      const int prev = atomicAdd(&p.ticket_rt[rt], 1);
      last = prev == sg - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    float y = 0.f;
    for (int q = 0; q < sg; ++q) y += ldcg_f32(p.ypart + (int64_t)q * p.H + rt * 32 + lane);
    if (p.down_bias) y += load_as_f32(p.down_bias, p.bias_dtype, rt * 32 + lane);
    store_from_f32(p.y, p.y_dtype, rt * 32 + lane, y);
    if (lane == 0) p.ticket_rt[rt] = 0;
  }
}

// ============================================================================
// host side
// ============================================================================
static int dtype_ok(int d) { return d == NSM_F32 || d == NSM_F16 || d == NSM_BF16; }

struct KernelSetup {
  bool done = false;
  int gateup_ctas_per_sm = 0;
  int down_ctas_per_sm = 0;
};
static KernelSetup g_setup[64];

static int setup_kernels(const DeviceInfo& d, KernelSetup** out) {
  KernelSetup& s = g_setup[d.device];
  if (!s.done) {
    const int smem = kLutBytes;
    NSM_CHECK_CUDA(cudaFuncSetAttribute(gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    NSM_CHECK_CUDA(cudaFuncSetAttribute(down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    NSM_CHECK_CUDA(cudaFuncSetAttribute(router_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kMaxNumBlocks * 8));
    NSM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&s.gateup_ctas_per_sm, gateup_kernel, 256, smem));
    NSM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&s.down_ctas_per_sm, down_kernel, 256, smem));
    if (s.gateup_ctas_per_sm <= 0 || s.down_ctas_per_sm <= 0) return fail(NSM_ERR_CUDA, "kernel occupancy is zero");
    s.done = true;
  }
  *out = &s;
  return NSM_OK;
}

struct MlpPlan {
  int H;
  int I;
  int k;
  const nsm_mlp_weights* w;
  const int* rows;
  const int* count;
  const int* row_block;
  int bias_by_block;
  const void* act_mask;
  int mask_dtype;
  float* act_out;
  void* y;
  int y_dtype;
  const float* norm_scale;
};

static int validate_weights(const nsm_mlp_weights* w, int H) {
  NSM_REQUIRE(w != nullptr, NSM_ERR_INVALID_ARG, "weights descriptor is NULL");
  NSM_REQUIRE(w->gate_packed && w->gate_absmax && w->up_packed && w->up_absmax && w->down_packed &&
                  w->down_absmax,
              NSM_ERR_INVALID_ARG, "a weight pointer is NULL");
  NSM_REQUIRE(w->gate_code && w->up_code && w->down_code, NSM_ERR_INVALID_ARG, "a code table pointer is NULL");
  NSM_REQUIRE(w->pool_rows > 0, NSM_ERR_INVALID_ARG, "pool_rows must be > 0");
  NSM_REQUIRE(((uintptr_t)w->gate_packed & 7) == 0 && ((uintptr_t)w->up_packed & 7) == 0, NSM_ERR_INVALID_ARG,
              "gate/up packed pointers must be 8-byte aligned");
  NSM_REQUIRE(((uintptr_t)w->down_packed & 3) == 0, NSM_ERR_INVALID_ARG, "down packed pointer must be 4-byte aligned");
  if (w->gate_bias || w->up_bias || w->down_bias)
    NSM_REQUIRE(dtype_ok(w->bias_dtype), NSM_ERR_INVALID_ARG, "bad bias dtype");
  const int64_t gs = w->gateup_block_stride ? w->gateup_block_stride : (int64_t)16 * H;
  NSM_REQUIRE(gs % 8 == 0, NSM_ERR_INVALID_ARG, "gate/up block stride must be a multiple of 8 bytes");
  const int64_t drs = w->down_row_stride ? w->down_row_stride : 16;
  const int64_t dbs = w->down_block_stride ? w->down_block_stride : (int64_t)16 * H;
  NSM_REQUIRE(drs % 4 == 0 && dbs % 4 == 0, NSM_ERR_INVALID_ARG, "down strides must be multiples of 4 bytes");
  return NSM_OK;
}

static int launch_mlp(const MlpPlan& m, const DecodeWs& ws, cudaStream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  KernelSetup* ks = nullptr;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  const nsm_mlp_weights* w = m.w;
  GateUpParams gp{};
  gp.gate = w->gate_packed;
  gp.gate_am = w->gate_absmax;
  gp.up = w->up_packed;
  gp.up_am = w->up_absmax;
  gp.gstride = w->gateup_block_stride ? w->gateup_block_stride : (int64_t)16 * m.H;
  gp.gastride = w->gateup_absmax_block_stride ? w->gateup_absmax_block_stride : (int64_t)m.H / 2;
  gp.gate_code = w->gate_code;
  gp.up_code = w->up_code;
  gp.gate_bias = w->gate_bias;
  gp.up_bias = w->up_bias;
  gp.bias_dtype = w->bias_dtype;
  gp.bias_by_block = m.bias_by_block;
  gp.H = m.H;
  gp.rows = m.rows;
  gp.count_ptr = m.count;
  gp.row_block = m.row_block;
  gp.x16 = ws.x16;
  gp.xscale = ws.xscale;
  gp.norm_scale = m.norm_scale;
  gp.act_mask = m.act_mask;
  gp.mask_dtype = m.mask_dtype;
  gp.gu_part = ws.gu_part;
  gp.ticket_slot = ws.ticket_slot;
  gp.act16 = ws.act16;
  gp.act_scale = ws.act_scale;
  gp.act_out = m.act_out;
  const int gu_ctas = dev.sm_count * ks->gateup_ctas_per_sm;
  gp.total_warps = gu_ctas * 8;
  gateup_kernel<<<gu_ctas, 256, kLutBytes, stream>>>(gp);
  NSM_CHECK_CUDA(cudaGetLastError());

  DownParams dp{};
  dp.down = w->down_packed;
  dp.down_am = w->down_absmax;
  const bool dflt = !w->down_block_stride && !w->down_row_stride && !w->down_absmax_block_stride &&
                    !w->down_absmax_row_stride;
  dp.dbs = dflt ? (int64_t)16 * m.H : w->down_block_stride;
  dp.drs = dflt ? 16 : w->down_row_stride;
  dp.dabs = dflt ? (int64_t)m.H : w->down_absmax_block_stride;
  dp.dars = dflt ? 1 : w->down_absmax_row_stride;
  dp.pair = w->down_absmax_pair;
  dp.down_code = w->down_code;
  dp.down_bias = w->down_bias;
  dp.bias_dtype = w->bias_dtype;
  dp.H = m.H;
  dp.rows = m.rows;
  dp.count_ptr = m.count;
  dp.act16 = ws.act16;
  dp.act_scale = ws.act_scale;
  dp.ypart = ws.ypart;
  dp.ticket_rt = ws.ticket_rowtile;
  dp.y = m.y;
  dp.y_dtype = m.y_dtype;
  const int dn_ctas = dev.sm_count * ks->down_ctas_per_sm;
  dp.total_warps = dn_ctas * 8;
  down_kernel<<<dn_ctas, 256, kLutBytes, stream>>>(dp);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

static int router_a_launch(const void* x, int x_dtype, const nsm_layer_io* io, const nsm_router_weights* rw, int H,
                           const DecodeWs& ws, cudaStream_t stream) {
  RouterAParams a{};
  a.x = x;
  a.x_dtype = x_dtype;
  if (io && io->residual) {
    a.residual = io->residual;
    a.y_prev = io->y_prev;
    a.y_prev_dtype = io->y_prev_dtype;
    a.norm_w = io->norm_weight;
    a.norm_w_dtype = io->norm_weight_dtype;
    a.eps = io->eps;
    a.use_norm = 1;
  }
  if (rw) {
    a.enc_w = rw->enc_w;
    a.enc_b = rw->enc_b;
    a.wdtype = rw->weight_dtype;
    a.rank = rw->rank;
    a.basis_top_k = rw->basis_top_k;
  }
  a.H = H;
  int ctas = std::min(kRouterMaxCtas, std::max(1, H / 64));
  int cpc = ((H + ctas - 1) / ctas + 63) / 64 * 64;
  // aim for ~128 columns per CTA (one wave of small CTAs)
  cpc = std::max(cpc, 128);
  ctas = (H + cpc - 1) / cpc;
  a.cols_per_cta = cpc;
  a.ws = ws;
  router_latent_kernel<<<ctas, 256, cpc * sizeof(float), stream>>>(a);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

static int validate_router(const nsm_router_weights* rw, int H) {
  NSM_REQUIRE(rw != nullptr, NSM_ERR_INVALID_ARG, "router weights are NULL");
  NSM_REQUIRE(rw->enc_w && rw->score_w, NSM_ERR_INVALID_ARG, "router enc_w/score_w is NULL");
  NSM_REQUIRE(dtype_ok(rw->weight_dtype), NSM_ERR_INVALID_ARG, "bad router weight dtype");
  NSM_REQUIRE(rw->rank > 0 && rw->rank <= kMaxRank, NSM_ERR_UNSUPPORTED, "router rank must be in [1, 256]");
  NSM_REQUIRE(rw->num_blocks > 0 && rw->num_blocks <= kMaxNumBlocks, NSM_ERR_UNSUPPORTED,
              "router num_blocks must be in [1, 8192]");
  NSM_REQUIRE(rw->top_k > 0, NSM_ERR_INVALID_ARG, "top_k must be > 0");
  (void)H;
  return NSM_OK;
}

static int router_b_launch(const nsm_router_weights* rw, int k, int32_t* idx_out, float* score_out,
                           float* latent_out, const nsm_block_map* map, int pool_rows, const DecodeWs& ws,
                           cudaStream_t stream) {
  RouterBParams b{};
  b.score_w = rw->score_w;
  b.score_b = rw->score_b;
  b.wdtype = rw->weight_dtype;
  b.dbn = rw->down_block_norm;
  b.legacy = rw->legacy_abs_latent;
  b.rank = rw->rank;
  b.NB = rw->num_blocks;
  b.top_k = k;
  int sn = 1;
  while (sn < b.NB) sn <<= 1;
  b.sort_n = sn;
  b.idx_out = idx_out;
  b.score_out = score_out;
  b.latent_out = latent_out;
  b.slot_of_block = map ? map->slot_of_block : nullptr;
  b.block_begin = map ? map->block_begin : 0;
  b.block_end = map ? map->block_end : b.NB;
  b.pool_rows = pool_rows;
  b.ws = ws;
  const int ctas = (b.NB + 511) / 512;
  router_select_kernel<<<ctas, 512, sn * 8, stream>>>(b);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

}  // namespace nsm

using namespace nsm;

extern "C" {

int nsm_route(const void* x, int32_t x_dtype, int32_t hidden, const nsm_router_weights* rw, int32_t* idx_out,
              float* score_out, float* latent_out, void* ws, size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  st = validate_router(rw, hidden);
  if (st) return st;
  NSM_REQUIRE(x != nullptr && dtype_ok(x_dtype), NSM_ERR_INVALID_ARG, "x is NULL or has a bad dtype");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0, NSM_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  NSM_REQUIRE(idx_out != nullptr, NSM_ERR_INVALID_ARG, "idx_out is NULL");
  const int k = std::max(1, std::min(rw->top_k, rw->num_blocks));
  NSM_REQUIRE(k <= kMaxTopK, NSM_ERR_UNSUPPORTED, "top_k too large");
  const int I = rw->num_blocks * 32;
  const size_t need = decode_ws_layout(nullptr, hidden, I, k, rw->rank).bytes;
  NSM_REQUIRE(ws != nullptr && ws_bytes >= need, NSM_ERR_WORKSPACE, "workspace too small for nsm_route");
  DecodeWs w = decode_ws_layout(ws, hidden, I, k, rw->rank);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  st = router_a_launch(x, x_dtype, nullptr, rw, hidden, w, s);
  if (st) return st;
  return router_b_launch(rw, k, idx_out, score_out, latent_out, nullptr, rw->num_blocks, w, s);
}

int nsm_sparse_mlp_decode(const void* x, int32_t x_dtype, int32_t hidden, int32_t intermediate,
                          const nsm_layer_io* io, const nsm_router_weights* rw, const int32_t* idx_in, int32_t k_in,
                          const nsm_block_map* map, const nsm_mlp_weights* w, void* y, int32_t y_dtype,
                          int32_t* idx_out, float* score_out, void* ws, size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0, NSM_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  NSM_REQUIRE(intermediate > 0 && intermediate % 64 == 0, NSM_ERR_UNSUPPORTED,
              "intermediate must be a positive multiple of 64");
  const bool resid = io != nullptr && io->residual != nullptr;
  NSM_REQUIRE(resid || (x != nullptr && dtype_ok(x_dtype)), NSM_ERR_INVALID_ARG, "x is NULL or has a bad dtype");
  if (resid && io->y_prev) NSM_REQUIRE(dtype_ok(io->y_prev_dtype), NSM_ERR_INVALID_ARG, "bad y_prev dtype");
  if (resid && io->norm_weight)
    NSM_REQUIRE(dtype_ok(io->norm_weight_dtype), NSM_ERR_INVALID_ARG, "bad norm weight dtype");
  NSM_REQUIRE(y != nullptr && dtype_ok(y_dtype), NSM_ERR_INVALID_ARG, "y is NULL or has a bad dtype");
  st = validate_weights(w, hidden);
  if (st) return st;
  const int NB = intermediate / 32;
  int k, rank = 1;
  if (idx_in != nullptr) {
    NSM_REQUIRE(k_in > 0, NSM_ERR_INVALID_ARG, "k_in must be > 0 with idx_in");
    k = k_in;
  } else {
    st = validate_router(rw, hidden);
    if (st) return st;
    NSM_REQUIRE(rw->num_blocks == NB, NSM_ERR_INVALID_ARG, "router num_blocks != intermediate/32");
    k = std::max(1, std::min(rw->top_k, NB));
    rank = rw->rank;
  }
  if (rw) rank = std::max(rank, rw->rank);
  NSM_REQUIRE(k <= kMaxTopK, NSM_ERR_UNSUPPORTED, "top_k too large");
  const size_t need = decode_ws_layout(nullptr, hidden, intermediate, k, rank).bytes;
  NSM_REQUIRE(ws != nullptr && ws_bytes >= need, NSM_ERR_WORKSPACE, "workspace too small for nsm_sparse_mlp_decode");
  DecodeWs wsl = decode_ws_layout(ws, hidden, intermediate, k, rank);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;

  st = router_a_launch(x, x_dtype, io, idx_in ? nullptr : rw, hidden, wsl, s);
  if (st) return st;
  if (idx_in == nullptr) {
    st = router_b_launch(rw, k, idx_out, score_out, nullptr, map, w->pool_rows, wsl, s);
    if (st) return st;
  } else {
    RouterBParams b{};
    b.NB = NB;
    b.slot_of_block = map ? map->slot_of_block : nullptr;
    b.block_begin = map ? map->block_begin : 0;
    b.block_end = map ? map->block_end : NB;
    b.pool_rows = w->pool_rows;
    b.ws = wsl;
    select_given_kernel<<<1, 512, 0, s>>>(b, idx_in, k);
    NSM_CHECK_CUDA(cudaGetLastError());
  }
  MlpPlan m{};
  m.H = hidden;
  m.I = intermediate;
  m.k = k;
  m.w = w;
  m.rows = wsl.rows;
  m.count = wsl.count;
  m.row_block = wsl.row_block;
  m.bias_by_block = 1;
  m.y = y;
  m.y_dtype = y_dtype;
  m.norm_scale = wsl.norm_scale;
  return launch_mlp(m, wsl, s);
}

int nsm_decode_gathered(const void* x, int32_t x_dtype, int32_t hidden, int32_t num_blocks_gathered,
                        const nsm_mlp_weights* w, void* y, int32_t y_dtype, float* act_out, void* ws,
                        size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0, NSM_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  NSM_REQUIRE(num_blocks_gathered > 0 && num_blocks_gathered <= kMaxTopK, NSM_ERR_UNSUPPORTED,
              "num_blocks_gathered must be in [1, 4096]");
  NSM_REQUIRE(x != nullptr && dtype_ok(x_dtype), NSM_ERR_INVALID_ARG, "x is NULL or has a bad dtype");
  NSM_REQUIRE(y != nullptr && dtype_ok(y_dtype), NSM_ERR_INVALID_ARG, "y is NULL or has a bad dtype");
  st = validate_weights(w, hidden);
  if (st) return st;
  NSM_REQUIRE(w->pool_rows >= num_blocks_gathered, NSM_ERR_INVALID_ARG, "pool_rows < num_blocks_gathered");
  const int k = num_blocks_gathered;
  const int I = 64 * ((k * 32 + 63) / 64);
  const size_t need = decode_ws_layout(nullptr, hidden, I, k, 1).bytes;
  NSM_REQUIRE(ws != nullptr && ws_bytes >= need, NSM_ERR_WORKSPACE, "workspace too small for nsm_decode_gathered");
  DecodeWs wsl = decode_ws_layout(ws, hidden, I, k, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  st = router_a_launch(x, x_dtype, nullptr, nullptr, hidden, wsl, s);
  if (st) return st;
  identity_rows_kernel<<<(k + 255) / 256, 256, 0, s>>>(wsl.rows, wsl.count, wsl.sel_idx, k);
  NSM_CHECK_CUDA(cudaGetLastError());
  MlpPlan m{};
  m.H = hidden;
  m.I = I;
  m.k = k;
  m.w = w;
  m.rows = wsl.rows;
  m.count = wsl.count;
  m.row_block = wsl.sel_idx;
  m.bias_by_block = 0;
  m.act_out = act_out;
  m.y = y;
  m.y_dtype = y_dtype;
  m.norm_scale = nullptr;
  return launch_mlp(m, wsl, s);
}

size_t nsm_decode_rows_workspace_bytes(int hidden, int num_blocks_gathered, int rows) {
  if (hidden <= 0 || num_blocks_gathered <= 0 || rows <= 0) return 0;
  const int I = 64 * ((num_blocks_gathered * 32 + 63) / 64);
  return decode_ws_layout(nullptr, hidden, I, num_blocks_gathered, 1).bytes;
}

int nsm_decode_gathered_rows(const void* x, int32_t x_dtype, int32_t rows, int32_t hidden,
                             int32_t num_blocks_gathered, const void* flat_mask, int32_t mask_dtype,
                             const nsm_mlp_weights* w, void* y, int32_t y_dtype, void* ws, size_t ws_bytes,
                             nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  NSM_REQUIRE(rows > 0, NSM_ERR_INVALID_ARG, "rows must be > 0");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0, NSM_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  NSM_REQUIRE(num_blocks_gathered > 0 && num_blocks_gathered <= kMaxTopK, NSM_ERR_UNSUPPORTED,
              "num_blocks_gathered must be in [1, 4096]");
  NSM_REQUIRE(x != nullptr && dtype_ok(x_dtype), NSM_ERR_INVALID_ARG, "x is NULL or has a bad dtype");
  NSM_REQUIRE(y != nullptr && dtype_ok(y_dtype), NSM_ERR_INVALID_ARG, "y is NULL or has a bad dtype");
  NSM_REQUIRE(flat_mask == nullptr || dtype_ok(mask_dtype), NSM_ERR_INVALID_ARG, "bad mask dtype");
  st = validate_weights(w, hidden);
  if (st) return st;
  const int k = num_blocks_gathered;
  const int I = 64 * ((k * 32 + 63) / 64);
  const size_t need = decode_ws_layout(nullptr, hidden, I, k, 1).bytes;
  NSM_REQUIRE(ws != nullptr && ws_bytes >= need, NSM_ERR_WORKSPACE, "workspace too small");
  DecodeWs wsl = decode_ws_layout(ws, hidden, I, k, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  identity_rows_kernel<<<(k + 255) / 256, 256, 0, s>>>(wsl.rows, wsl.count, wsl.sel_idx, k);
  NSM_CHECK_CUDA(cudaGetLastError());
  const int xes = x_dtype == NSM_F32 ? 4 : 2;
  const int yes = y_dtype == NSM_F32 ? 4 : 2;
  const int mes = mask_dtype == NSM_F32 ? 4 : 2;
  for (int r = 0; r < rows; ++r) {
    st = router_a_launch(reinterpret_cast<const char*>(x) + (size_t)r * hidden * xes, x_dtype, nullptr, nullptr,
                         hidden, wsl, s);
    if (st) return st;
    MlpPlan m{};
    m.H = hidden;
    m.I = I;
    m.k = k;
    m.w = w;
    m.rows = wsl.rows;
    m.count = wsl.count;
    m.row_block = wsl.sel_idx;
    m.bias_by_block = 0;
    m.act_mask = flat_mask ? reinterpret_cast<const char*>(flat_mask) + (size_t)r * k * 32 * mes : nullptr;
    m.mask_dtype = mask_dtype;
    m.y = reinterpret_cast<char*>(y) + (size_t)r * hidden * yes;
    m.y_dtype = y_dtype;
    m.norm_scale = nullptr;
    st = launch_mlp(m, wsl, s);
    if (st) return st;
  }
  return NSM_OK;
}

}  // extern "C"
