// nsm_union.cu -- multi-token decode over the union of the tokens' selected
// blocks (up to 32 tokens), on the tensor cores.
//
// The reference handles rows > 1 by gathering the union of the rows' blocks
// once (_build_sparse_active_layout, streaming_llama_runtime.py:4857-4908:
// union in ascending block order, per-row flat_mask) and running the fallback
// math on it (:5433-5492): g = x W_g^T * mask, u = x W_u^T * mask,
// act = silu(g) * u, y = act W_d^T.  Here every 64-column NF4 tile of a union
// block is dequantised once and multiplied against all tokens with
// mma.sync.m16n8k16 (4 token groups of 8), so the weight bytes are read once
// per union block instead of once per token.
//
//   union_build_kernel     one CTA: per-block row bitmasks, ascending union of
//                          the blocks present in the pool, per-slot row masks.
//   union_x_kernel         fp16 copy of each token's x with one power-of-two
//                          scale per token (exact for bf16 inputs).
//   union_gateup_kernel    warps stream balanced ranges of (union slot, tile)
//                          pairs; fp32 partials per slot segment.
//   union_act_kernel       per slot: fixed-order segment sums, token scale,
//                          row mask, SiLU(g)*u -> fp16 with one power-of-two
//                          scale per (slot, token).
//   union_down_kernel      CTA = (slot range, range of 64-row groups): the slot
//                          range's activations staged in shared memory, each
//                          warp streams its 64-row groups over the slots with
//                          register-prefetched weights; partials per slot range.
//   union_y_kernel         fixed-order sums over the slot ranges -> y[token][h].
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "nsm.h"
#include "nsm_common.cuh"
#include "nsm_internal.h"
#include "nsm_nf4.cuh"

namespace nsm {

constexpr int kUnionRows = 32;       // tokens per call (4 groups of 8)
constexpr int kUnionGuMaxSeg = 6;    // gate/up partial segments per union slot
// down: slot ranges (= partial segments of y) and their size
constexpr int kUdMinSlots = 32;      // slots per range at least (unions up to 32 x 24 slots: 24 ranges)
constexpr int kUdMaxRanges = 24;     // ranges for unions up to kUdMaxRanges x kUdMaxSlots slots
constexpr int kUdMaxSlots = 72;      // slots per range at most (their activations fill shared memory)
constexpr int kUnionThreads = 256;

struct UnionWs {
  int* err;
  __half* x16;      // [32][H]
  float* xscale;    // [32]
  int* u_rows;      // [Umax] pool rows of the union slots
  int* u_block;     // [Umax] block ids
  uint32_t* u_mask; // [Umax] bit r: token r selected the block
  int* u_count;     // [1]
  float* gu_part;   // [Umax][seg][2][32 tokens][32 rows]
  __half* act16;    // [Umax][32 tokens][32 cols]
  float* act_scale; // [Umax][32 tokens]
  float* ypart;     // [seg][H][32 tokens]
  size_t bytes;
};

static UnionWs union_ws_layout(void* base, int H, int umax) {
  UnionWs w{};
  char* b = reinterpret_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = b ? b + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  // the counter head of every workspace (nsm_workspace_error reads the error word there)
  int* head = reinterpret_cast<int*>(take((size_t)kCounterInts * sizeof(int)));
  w.err = head ? head + 2 : nullptr;
  w.x16 = reinterpret_cast<__half*>(take((size_t)kUnionRows * H * sizeof(__half)));
  w.xscale = reinterpret_cast<float*>(take(kUnionRows * sizeof(float)));
  w.u_rows = reinterpret_cast<int*>(take((size_t)umax * sizeof(int)));
  w.u_block = reinterpret_cast<int*>(take((size_t)umax * sizeof(int)));
  w.u_mask = reinterpret_cast<uint32_t*>(take((size_t)umax * sizeof(uint32_t)));
  w.u_count = reinterpret_cast<int*>(take(sizeof(int)));
  w.gu_part = reinterpret_cast<float*>(take((size_t)umax * kUnionGuMaxSeg * 2 * kUnionRows * 32 * sizeof(float)));
  w.act16 = reinterpret_cast<__half*>(take((size_t)umax * kUnionRows * 32 * sizeof(__half)));
  w.act_scale = reinterpret_cast<float*>(take((size_t)umax * kUnionRows * sizeof(float)));
  const int nseg = std::max(kUdMaxRanges, (umax + kUdMaxSlots - 1) / kUdMaxSlots);
  w.ypart = reinterpret_cast<float*>(take((size_t)nseg * H * kUnionRows * sizeof(float)));
  w.bytes = off;
  return w;
}

// ---------------------------------------------------------------------------
// union build
// ---------------------------------------------------------------------------
struct UnionBuildParams {
  const int32_t* idx;  // [rows][k]
  int rows, k, NB;
  const int32_t* slot_of_block;
  int block_begin, block_end, pool_rows;
  UnionWs ws;
  int32_t* union_out;  // optional [Umax] block ids
};

__device__ __forceinline__ int union_map_block(const UnionBuildParams& p, int b) {
  if (b < 0 || b >= p.NB) return -1;
  const int r = p.slot_of_block ? p.slot_of_block[b] : ((b >= p.block_begin && b < p.block_end) ? b - p.block_begin : -1);
  return (r >= 0 && r < p.pool_rows) ? r : -1;
}

// Block-wide exclusive scan of one int per thread (blockDim a multiple of 32, <= 1024).
__device__ __forceinline__ int union_scan(int v, int* total) {
  __shared__ int wsum[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
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
    if (lane < nw) wsum[lane] = s;
  }
  __syncthreads();
  const int before = (warp > 0 ? wsum[warp - 1] : 0) + x - v;
  *total = wsum[nw - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(1024) union_build_kernel(UnionBuildParams p) {
  extern __shared__ uint32_t rowbits[];  // [NB]
  pdl_trigger();
  pdl_wait();
  for (int b = threadIdx.x; b < p.NB; b += blockDim.x) rowbits[b] = 0u;
  __syncthreads();
  const int nidx = p.rows * p.k;
  for (int i0 = 0; i0 < nidx; i0 += 8 * (int)blockDim.x) {
    int bv[8];  // 8 loads in flight per thread
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * (int)blockDim.x + (int)threadIdx.x;
      bv[u] = i < nidx ? p.idx[i] : -1;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * (int)blockDim.x + (int)threadIdx.x;
      if (bv[u] >= 0 && bv[u] < p.NB) atomicOr(&rowbits[bv[u]], 1u << (i / p.k));
    }
  }
  __syncthreads();
  // ascending compaction of the selected blocks present in the pool
  const int per = (p.NB + blockDim.x - 1) / blockDim.x;
  const int lo = min(p.NB, (int)threadIdx.x * per), hi = min(p.NB, lo + per);
  int n = 0;
  for (int b = lo; b < hi; ++b) n += rowbits[b] != 0u && union_map_block(p, b) >= 0;
  int total;
  int pos = union_scan(n, &total);
  for (int b = lo; b < hi; ++b) {
    const uint32_t m = rowbits[b];
    if (m == 0u) continue;
    const int r = union_map_block(p, b);
    if (r < 0) continue;
    p.ws.u_rows[pos] = r;
    p.ws.u_block[pos] = b;
    p.ws.u_mask[pos] = m;
    if (p.union_out) p.union_out[pos] = b;
    ++pos;
  }
  if (threadIdx.x == 0) *p.ws.u_count = total;
}

// ---------------------------------------------------------------------------
// token prep
// ---------------------------------------------------------------------------
// One CTA per token: the row's values stay in registers between the max and
// the conversion (16 per thread at H <= 16384; longer rows are read twice).
constexpr int kUxThreads = 1024, kUxPer = 16;
__global__ void __launch_bounds__(kUxThreads) union_x_kernel(const void* x, int x_dtype, int rows, int H, UnionWs ws) {
  __shared__ float red[kUxThreads / 32];
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x;
  const int64_t base = (int64_t)r * H;
  float v[kUxPer];
  float m = 0.f;
  for (int c0 = 0; c0 < H; c0 += kUxThreads * kUxPer) {
#pragma unroll
    for (int i = 0; i < kUxPer; ++i) {
      const int c = c0 + i * kUxThreads + threadIdx.x;
      v[i] = (r < rows && c < H) ? load_as_f32(x, x_dtype, base + c) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < kUxPer; ++i) m = fmaxf(m, fabsf(v[i]));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float mm = 0.f;
  for (int w = 0; w < kUxThreads / 32; ++w) mm = fmaxf(mm, red[w]);
  const float sc = pow2_scale_for(mm);
  const float inv = 1.f / sc;
  for (int c0 = 0; c0 < H; c0 += kUxThreads * kUxPer) {
    if (H > kUxThreads * kUxPer) {  // reload (the registers hold the last chunk only)
#pragma unroll
      for (int i = 0; i < kUxPer; ++i) {
        const int c = c0 + i * kUxThreads + threadIdx.x;
        v[i] = (r < rows && c < H) ? load_as_f32(x, x_dtype, base + c) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < kUxPer; ++i) {
      const int c = c0 + i * kUxThreads + threadIdx.x;
      if (c < H) ws.x16[base + c] = __float2half_rn(v[i] * inv);
    }
  }
  if (threadIdx.x == 0) ws.xscale[r] = r < rows ? sc : 1.f;
}

// ---------------------------------------------------------------------------
// gate/up over the union
// ---------------------------------------------------------------------------
struct UnionMlpParams {
  const uint8_t* gate;
  const float* gate_am;
  const uint8_t* up;
  const float* up_am;
  int64_t gstride, gastride;
  const uint8_t* down;
  const float* down_am;
  int64_t dbs, dabs;
  const float* gate_code;
  const float* up_code;
  const float* down_code;
  int H, rows;
  int total_warps;
  UnionWs ws;
  void* y;
  int y_dtype;
};

struct UTile {
  uint4 w[2][2];  // [proj][row group]
  float4 am[2];
};

__device__ __forceinline__ void union_tile_load(const UnionMlpParams& p, int prow, int j, int lane, UTile& t) {
  const int g = lane >> 2;
  const uint8_t* gb = p.gate + (int64_t)prow * p.gstride;
  const uint8_t* ub = p.up + (int64_t)prow * p.gstride;
  const int64_t off = (int64_t)j * 1024 + lane * 16;
  t.w[0][0] = ldg_stream_u4(gb + off);
  t.w[0][1] = ldg_stream_u4(gb + off + 512);
  t.w[1][0] = ldg_stream_u4(ub + off);
  t.w[1][1] = ldg_stream_u4(ub + off + 512);
  t.am[0] = ldg_f4(p.gate_am + (int64_t)prow * p.gastride + j * 32 + g * 4);
  t.am[1] = ldg_f4(p.up_am + (int64_t)prow * p.gastride + j * 32 + g * 4);
}

// acc[proj][rg][grp][4]: rows (16rg+g, 16rg+g+8) x tokens (8grp+2t, 8grp+2t+1)
template <int kBase>
__device__ __forceinline__ void union_tile_mma(const UTile& tile, const uint32_t xb[4][8], uint32_t lb,
                                               float acc[2][2][4][4]) {
#pragma unroll
  for (int pr = 0; pr < 2; ++pr) {
#pragma unroll
    for (int rg = 0; rg < 2; ++rg) {
      const uint4 w = tile.w[pr][rg];
      uint32_t a[4][4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t lo = s < 2 ? w.x : w.y, hi = s < 2 ? w.z : w.w;
        const int kb = (s & 1) * 2;
        a[s][0] = lut_get<kBase>(lo, lb, kb, pr);
        a[s][1] = lut_get<kBase>(hi, lb, kb, pr);
        a[s][2] = lut_get<kBase>(lo, lb, kb + 1, pr);
        a[s][3] = lut_get<kBase>(hi, lb, kb + 1, pr);
      }
      const float am0 = rg ? tile.am[pr].z : tile.am[pr].x, am1 = rg ? tile.am[pr].w : tile.am[pr].y;
#pragma unroll
      for (int grp = 0; grp < 4; ++grp) {
        float d[4];
        mma_16816_z(d, a[0][0], a[0][1], a[0][2], a[0][3], xb[grp][0], xb[grp][1]);
        mma_16816(d, a[1][0], a[1][1], a[1][2], a[1][3], xb[grp][2], xb[grp][3]);
        mma_16816(d, a[2][0], a[2][1], a[2][2], a[2][3], xb[grp][4], xb[grp][5]);
        mma_16816(d, a[3][0], a[3][1], a[3][2], a[3][3], xb[grp][6], xb[grp][7]);
        acc[pr][rg][grp][0] = fmaf(d[0], am0, acc[pr][rg][grp][0]);
        acc[pr][rg][grp][1] = fmaf(d[1], am0, acc[pr][rg][grp][1]);
        acc[pr][rg][grp][2] = fmaf(d[2], am1, acc[pr][rg][grp][2]);
        acc[pr][rg][grp][3] = fmaf(d[3], am1, acc[pr][rg][grp][3]);
      }
    }
  }
}

template <int kBase>
__device__ __forceinline__ void union_gateup_body(const UnionMlpParams& p, uint32_t lb, int count) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int tpr = p.H >> 6;
  const int total = count * tpr;
  if (total == 0) return;
  const int nw = stream_warps(count, tpr, kUnionGuMaxSeg, p.total_warps);
  if (warp_global >= nw) return;
  const int q0 = stream_begin(total, nw, warp_global), q1 = stream_begin(total, nw, warp_global + 1);
  int s = q0 / tpr, j = q0 - s * tpr;
  int seg = warp_global - stream_owner(total, nw, s * tpr);
  float acc[2][2][4][4];
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int d = 0; d < 4; ++d) acc[a][b][c][d] = 0.f;
  // register double buffer: the next tile's weights and x fragments are in
  // flight while this tile's MMAs run
  UTile cur, nxt;
  uint4 xc[4][2], xn[4][2];
  auto load_x = [&](int jj, uint4 (&xf)[4][2]) {
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      const __half* xr = p.ws.x16 + (int64_t)(grp * 8 + g) * p.H + jj * 64 + t * 16;
      xf[grp][0] = ldg_u4(xr);
      xf[grp][1] = ldg_u4(xr + 8);
    }
  };
  int prow = __ldcg(p.ws.u_rows + s);
  union_tile_load(p, prow, j, lane, cur);
  load_x(j, xc);
  for (int q = q0; q < q1; ++q) {
    int sn = s, jn = j + 1;
    if (jn == tpr) { jn = 0; ++sn; }
    int prow_n = prow;
    if (q + 1 < q1) {
      if (sn != s) prow_n = __ldcg(p.ws.u_rows + sn);
      union_tile_load(p, prow_n, jn, lane, nxt);
      load_x(jn, xn);
    }
    uint32_t xb[4][8];
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      xb[grp][0] = xc[grp][0].x; xb[grp][1] = xc[grp][0].y; xb[grp][2] = xc[grp][0].z; xb[grp][3] = xc[grp][0].w;
      xb[grp][4] = xc[grp][1].x; xb[grp][5] = xc[grp][1].y; xb[grp][6] = xc[grp][1].z; xb[grp][7] = xc[grp][1].w;
    }
    union_tile_mma<kBase>(cur, xb, lb, acc);
    if (q + 1 == q1 || sn != s) {
      // partial of slot s, segment seg: [2][32 tokens][32 rows]
      float* part = p.ws.gu_part + ((int64_t)s * kUnionGuMaxSeg + seg) * (2 * kUnionRows * 32);
#pragma unroll
      for (int pr = 0; pr < 2; ++pr)
#pragma unroll
        for (int rg = 0; rg < 2; ++rg)
#pragma unroll
          for (int grp = 0; grp < 4; ++grp)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int row = rg * 16 + g + (e >> 1) * 8, tok = grp * 8 + 2 * t + (e & 1);
              part[(pr * kUnionRows + tok) * 32 + row] = acc[pr][rg][grp][e];
              acc[pr][rg][grp][e] = 0.f;
            }
      seg = 0;
    }
    s = sn;
    j = jn;
    prow = prow_n;
    cur = nxt;
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      xc[grp][0] = xn[grp][0];
      xc[grp][1] = xn[grp][1];
    }
  }
}

__global__ void __launch_bounds__(kUnionThreads, 1) union_gateup_kernel(UnionMlpParams p) {
  pdl_trigger();
  build_lut_dyn(p.gate_code, p.up_code);
  pdl_wait();
  __syncthreads();
  const int count = __ldcg(p.ws.u_count);
  const uint32_t lb = (threadIdx.x & 31) * 4u;
  if (lut_base_addr() == 0x400u)
    union_gateup_body<0x400>(p, lb, count);
  else
    union_gateup_body<-1>(p, lb, count);
}

// One CTA of 1024 threads per union slot: warp = token, lane = row.
__global__ void __launch_bounds__(1024) union_act_kernel(UnionMlpParams p) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x;
  const int count = __ldcg(p.ws.u_count);
  if (s >= count) return;
  const int tok = threadIdx.x >> 5, row = threadIdx.x & 31;
  const int tpr = p.H >> 6, total = count * tpr;
  const int nw = stream_warps(count, tpr, kUnionGuMaxSeg, p.total_warps);
  const int nseg = stream_owner(total, nw, s * tpr + tpr - 1) - stream_owner(total, nw, s * tpr) + 1;
  const float* base = p.ws.gu_part + (int64_t)s * kUnionGuMaxSeg * (2 * kUnionRows * 32);
  float g = 0.f, u = 0.f;
  float vg[kUnionGuMaxSeg], vu[kUnionGuMaxSeg];  // all segment loads in flight, summed in order
#pragma unroll
  for (int q = 0; q < kUnionGuMaxSeg; ++q) {
    vg[q] = q < nseg ? __ldcg(base + ((int64_t)q * 2 * kUnionRows + tok) * 32 + row) : 0.f;
    vu[q] = q < nseg ? __ldcg(base + ((int64_t)q * 2 * kUnionRows + kUnionRows + tok) * 32 + row) : 0.f;
  }
#pragma unroll
  for (int q = 0; q < kUnionGuMaxSeg; ++q)
    if (q < nseg) {
      g += vg[q];
      u += vu[q];
    }
  const float xs = __ldcg(p.ws.xscale + tok);
  g *= xs;
  u *= xs;
  const bool on = tok < p.rows && ((__ldcg(p.ws.u_mask + s) >> tok) & 1u);
  const float act = on ? silu_f32(g) * u : 0.f;
  const float m = warp_max(fabsf(act));
  const float sc = pow2_scale_for(m);
  p.ws.act16[((int64_t)s * kUnionRows + tok) * 32 + row] = __float2half_rn(act * (1.f / sc));
  if (row == 0) p.ws.act_scale[(int64_t)s * kUnionRows + tok] = sc;
}

// ---------------------------------------------------------------------------
// down over the union
// ---------------------------------------------------------------------------
// y[h][tok] = sum over slots s and their 32 columns c of W_d[h][s, c] act[s][tok][c].
// The slots split into nsr ranges (a function of the union's size only, so the
// y kernel finds the same split); a CTA takes one (slot range, range of 64-row
// groups) item, stages the range's activations (fp16 [tok][col] per slot, 2 KB)
// and their scales in shared memory, and each warp streams its 64-row groups
// over the range's slots: the weight pair (64 rows x 32 columns, 1 KB + the
// rows' absmax) comes from global memory kUdDepth pairs ahead in registers,
// the activation fragments from shared memory, 32 mma.sync per pair (2 row
// tiles x 2 row groups x 4 token groups x 2 K steps).  A warp owns whole row
// groups, so each (range, row group) partial is written once.
constexpr int kUdThreads = 256;
constexpr int kUdWarps = kUdThreads / 32;
constexpr int kUdDepth = 3;  // weight pairs in flight per warp, beyond the one computed
constexpr int kUdActOff = kSmemHead;                                      // [kUdMaxSlots][32 tok][32 col] fp16
constexpr int kUdScaleOff = kUdActOff + kUdMaxSlots * kUnionRows * 64;   // [kUdMaxSlots][32 tok] fp32
constexpr int kUdRowsOff = kUdScaleOff + kUdMaxSlots * kUnionRows * 4;   // [kUdMaxSlots] pool rows
constexpr int kUdSmem = kUdRowsOff + kUdMaxSlots * 4;
static_assert(kUdSmem <= 227 * 1024, "union down shared memory");

// Slot ranges of a union of `count` slots: at least kUdMinSlots slots per
// range, at most kUdMaxRanges ranges unless a range would pass kUdMaxSlots.
__device__ __forceinline__ int union_down_ranges(int count) {
  int n = (count + kUdMinSlots - 1) / kUdMinSlots;
  n = n < 1 ? 1 : (n > kUdMaxRanges ? kUdMaxRanges : n);
  const int need = (count + kUdMaxSlots - 1) / kUdMaxSlots;
  return n > need ? n : need;
}

struct UdPair {
  uint4 w0, w1;    // row tiles 0 and 1 of the 64-row group: rows g, g+8, 16+g, 24+g (.x .y .z .w), bytes 4t..4t+3
  float4 a0, a1;   // their absmax
};

template <int kBase>
__device__ __forceinline__ void union_down_pair(const UdPair& pr, uint32_t lb, const uint4 bf[4], const float2 as[4],
                                                float (&acc)[2][2][4][4]) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4 w = r ? pr.w1 : pr.w0;
    const float4 am = r ? pr.a1 : pr.a0;
#pragma unroll
    for (int rg = 0; rg < 2; ++rg) {
      const uint32_t w0 = rg ? w.z : w.x, w1 = rg ? w.w : w.y;
      const uint32_t a00 = lut_get<kBase>(w0, lb, 0, 0), a01 = lut_get<kBase>(w1, lb, 0, 0);
      const uint32_t a02 = lut_get<kBase>(w0, lb, 1, 0), a03 = lut_get<kBase>(w1, lb, 1, 0);
      const uint32_t a10 = lut_get<kBase>(w0, lb, 2, 0), a11 = lut_get<kBase>(w1, lb, 2, 0);
      const uint32_t a12 = lut_get<kBase>(w0, lb, 3, 0), a13 = lut_get<kBase>(w1, lb, 3, 0);
      const float r0 = rg ? am.z : am.x, r1 = rg ? am.w : am.y;
#pragma unroll
      for (int grp = 0; grp < 4; ++grp) {
        float d[4];
        mma_16816_z(d, a00, a01, a02, a03, bf[grp].x, bf[grp].y);
        mma_16816(d, a10, a11, a12, a13, bf[grp].z, bf[grp].w);
        acc[r][rg][grp][0] = fmaf(d[0], r0 * as[grp].x, acc[r][rg][grp][0]);
        acc[r][rg][grp][1] = fmaf(d[1], r0 * as[grp].y, acc[r][rg][grp][1]);
        acc[r][rg][grp][2] = fmaf(d[2], r1 * as[grp].x, acc[r][rg][grp][2]);
        acc[r][rg][grp][3] = fmaf(d[3], r1 * as[grp].y, acc[r][rg][grp][3]);
      }
    }
  }
}

template <int kBase>
__device__ __forceinline__ void union_down_body(const UnionMlpParams& p, uint32_t lb, int count) {
  char* smem = reinterpret_cast<char*>(g_lut_smem);
  const __half* sact = reinterpret_cast<const __half*>(smem + kUdActOff);
  const float* sscale = reinterpret_cast<const float*>(smem + kUdScaleOff);
  int* srows = reinterpret_cast<int*>(smem + kUdRowsOff);
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, warp = threadIdx.x >> 5;
  const int RP = p.H >> 6;
  const int nsr = union_down_ranges(count);
  const int per = (count + nsr - 1) / nsr;
  const int nrr = max(1, (int)gridDim.x / nsr);
  for (int item = blockIdx.x; item < nsr * nrr; item += gridDim.x) {
    const int sr = item / nrr, rr = item - sr * nrr;
    const int s0 = sr * per, s1 = min(count, s0 + per), ns = s1 - s0;
    const int rp0 = (int)((int64_t)RP * rr / nrr), rp1 = (int)((int64_t)RP * (rr + 1) / nrr);
    __syncthreads();  // the previous item's readers are done with the staging buffers
    if (ns > 0) {
      const uint4* src = reinterpret_cast<const uint4*>(p.ws.act16 + (int64_t)s0 * kUnionRows * 32);
      uint4* dst = reinterpret_cast<uint4*>(smem + kUdActOff);
      for (int i = threadIdx.x; i < ns * kUnionRows * 4; i += blockDim.x) dst[i] = __ldcg(src + i);
      float* ssc = reinterpret_cast<float*>(smem + kUdScaleOff);
      for (int i = threadIdx.x; i < ns * kUnionRows; i += blockDim.x)
        ssc[i] = __ldcg(p.ws.act_scale + (int64_t)s0 * kUnionRows + i);
      for (int i = threadIdx.x; i < ns; i += blockDim.x) srows[i] = __ldcg(p.ws.u_rows + s0 + i);
    }
    __syncthreads();
    if (ns <= 0) continue;
    // this warp's row groups: rp0 + warp, rp0 + warp + kUdWarps, ...
    const int nmine = rp1 - rp0 > warp ? (rp1 - rp0 - warp + kUdWarps - 1) / kUdWarps : 0;
    const int npairs = nmine * ns;
    if (npairs == 0) continue;
    int lrp = rp0 + warp, ls = 0;  // load cursor
    auto load = [&](UdPair& pr) {
      const int64_t prow = srows[ls];
      const uint8_t* wb = p.down + prow * p.dbs + (int64_t)lrp * 1024 + lane * 16;
      pr.w0 = ldg_stream_u4(wb);
      pr.w1 = ldg_stream_u4(wb + 512);
      const float* ab = p.down_am + prow * p.dabs + lrp * 64 + g * 4;
      pr.a0 = ldg_f4(ab);
      pr.a1 = ldg_f4(ab + 32);
      if (++ls == ns) {
        ls = 0;
        lrp += kUdWarps;
      }
    };
    UdPair buf[kUdDepth + 1];
#pragma unroll
    for (int i = 0; i < kUdDepth + 1; ++i)
      if (i < npairs) load(buf[i]);
    float acc[2][2][4][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int b2 = 0; b2 < 2; ++b2)
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int d = 0; d < 4; ++d) acc[a][b2][c][d] = 0.f;
    int rp = rp0 + warp, s = 0;
    for (int q0 = 0; q0 < npairs; q0 += kUdDepth + 1) {
#pragma unroll
      for (int u = 0; u < kUdDepth + 1; ++u) {
        const int q = q0 + u;
        if (q >= npairs) break;
        const UdPair cur = buf[u];
        if (q + kUdDepth + 1 < npairs) load(buf[u]);
        uint4 bf[4];
        float2 as[4];
#pragma unroll
        for (int grp = 0; grp < 4; ++grp) {
          bf[grp] = *reinterpret_cast<const uint4*>(sact + ((s * kUnionRows + grp * 8 + g) * 32 + t * 8));
          as[grp] = *reinterpret_cast<const float2*>(sscale + s * kUnionRows + grp * 8 + 2 * t);
        }
        union_down_pair<kBase>(cur, lb, bf, as, acc);
        if (++s == ns) {
          // row group rp done: its partial for this slot range
          float* yp = p.ws.ypart + ((int64_t)sr * p.H + (int64_t)rp * 64) * kUnionRows;
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int rg = 0; rg < 2; ++rg)
#pragma unroll
              for (int grp = 0; grp < 4; ++grp)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int row = r * 32 + rg * 16 + g + (e >> 1) * 8, tok = grp * 8 + 2 * t + (e & 1);
                  yp[row * kUnionRows + tok] = acc[r][rg][grp][e];
                  acc[r][rg][grp][e] = 0.f;
                }
          s = 0;
          rp += kUdWarps;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kUdThreads, 1) union_down_kernel(UnionMlpParams p) {
  pdl_trigger();
  build_lut_dyn(p.down_code, p.down_code);
  pdl_wait();
  __syncthreads();
  const int count = __ldcg(p.ws.u_count);
  const uint32_t lb = (threadIdx.x & 31) * 4u;
  if (lut_base_addr() == 0x400u)
    union_down_body<0x400>(p, lb, count);
  else
    union_down_body<-1>(p, lb, count);
}

// y[token][h] = the slot ranges' partials summed in range order; one thread per (h, token).
__global__ void __launch_bounds__(256) union_y_kernel(UnionMlpParams p) {
  pdl_trigger();
  pdl_wait();
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = e / kUnionRows, tok = e % kUnionRows;
  if (h >= p.H) return;
  const int count = __ldcg(p.ws.u_count);
  float y = 0.f;
  if (count > 0) {
    const int nseg = union_down_ranges(count);
    for (int q0 = 0; q0 < nseg; q0 += 8) {
      float v[8];  // eight segment loads in flight, summed in order
#pragma unroll
      for (int u = 0; u < 8; ++u)
        v[u] = q0 + u < nseg ? __ldcg(p.ws.ypart + ((int64_t)(q0 + u) * p.H + h) * kUnionRows + tok) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (q0 + u < nseg) y += v[u];
    }
  }
  if (tok < p.rows) store_from_f32(p.y, p.y_dtype, (int64_t)tok * p.H + h, y);
}

static int union_setup(int device, int* gu_ctas, int* dn_ctas) {
  static int cache[64][2];
  static bool done[64] = {};
  if (device < 0 || device >= 64) return fail(NSM_ERR_DEVICE, "device index out of range");
  if (!done[device]) {
    NSM_CHECK_CUDA(cudaFuncSetAttribute(union_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kMaxNumBlocks * 4));
    NSM_CHECK_CUDA(cudaFuncSetAttribute(union_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemHead));
    NSM_CHECK_CUDA(cudaFuncSetAttribute(union_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kUdSmem));
    NSM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&cache[device][0], union_gateup_kernel,
                                                                 kUnionThreads, kSmemHead));
    NSM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&cache[device][1], union_down_kernel,
                                                                 kUdThreads, kUdSmem));
    if (cache[device][0] <= 0 || cache[device][1] <= 0) return fail(NSM_ERR_CUDA, "union kernel occupancy is zero");
    done[device] = true;
  }
  *gu_ctas = cache[device][0];
  *dn_ctas = cache[device][1];
  return NSM_OK;
}

}  // namespace nsm

using namespace nsm;

extern "C" {

size_t nsm_union_workspace_bytes(int hidden, int intermediate, int rows, int k) {
  if (hidden <= 0 || intermediate <= 0 || rows <= 0 || k <= 0) return 0;
  const int umax = std::min(intermediate / 32, rows * k);
  return union_ws_layout(nullptr, hidden, umax).bytes;
}

int nsm_union_decode(const void* x, int32_t x_dtype, int32_t rows, int32_t hidden, int32_t intermediate,
                     const int32_t* idx, int32_t k, const nsm_block_map* map, const nsm_mlp_weights* w, void* y,
                     int32_t y_dtype, int32_t* union_out, int32_t* union_count_out, void* ws, size_t ws_bytes,
                     nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  auto dtype_ok = [](int d) { return d == NSM_F32 || d == NSM_F16 || d == NSM_BF16; };
  NSM_REQUIRE(rows > 0 && rows <= kUnionRows, NSM_ERR_UNSUPPORTED, "rows must be in [1, 32]");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
  NSM_REQUIRE(intermediate > 0 && intermediate % 64 == 0 && intermediate / 32 <= kMaxNumBlocks, NSM_ERR_UNSUPPORTED,
              "intermediate must be a positive multiple of 64 with at most 8192 blocks");
  NSM_REQUIRE(k > 0, NSM_ERR_INVALID_ARG, "k must be > 0");
  NSM_REQUIRE(x && idx && w && y, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(dtype_ok(x_dtype) && dtype_ok(y_dtype), NSM_ERR_INVALID_ARG, "bad x or y dtype");
  const int tiled = NSM_LAYOUT_GATEUP_TILED | NSM_LAYOUT_DOWN_TILED;
  NSM_REQUIRE((w->layout & tiled) == tiled, NSM_ERR_UNSUPPORTED,
              "the union decode reads tiled gate/up and down pools");
  NSM_REQUIRE(!w->gate_bias && !w->up_bias && !w->down_bias, NSM_ERR_UNSUPPORTED,
              "the union decode does not take biases");
  NSM_REQUIRE(w->gate_packed && w->gate_absmax && w->up_packed && w->up_absmax && w->down_packed &&
                  w->down_absmax && w->gate_code && w->up_code && w->down_code && w->pool_rows > 0,
              NSM_ERR_INVALID_ARG, "incomplete weights descriptor");
  NSM_REQUIRE(((uintptr_t)w->gate_packed | (uintptr_t)w->up_packed | (uintptr_t)w->down_packed |
               (uintptr_t)w->gate_absmax | (uintptr_t)w->up_absmax | (uintptr_t)w->down_absmax) % 16 == 0,
              NSM_ERR_INVALID_ARG, "pool pointers must be 16-byte aligned");
  const int NB = intermediate / 32;
  const int umax = std::min(NB, rows * k);
  const size_t need = union_ws_layout(nullptr, hidden, umax).bytes;
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "nsm_union_decode: workspace missing, not 256-byte aligned or too small");
  UnionWs wsl = union_ws_layout(ws, hidden, umax);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int gu_per_sm, dn_per_sm;
  st = union_setup(dev.device, &gu_per_sm, &dn_per_sm);
  if (st) return st;

  UnionBuildParams bp{};
  bp.idx = idx;
  bp.rows = rows;
  bp.k = k;
  bp.NB = NB;
  bp.slot_of_block = map ? map->slot_of_block : nullptr;
  bp.block_begin = map ? map->block_begin : 0;
  bp.block_end = map ? map->block_end : NB;
  bp.pool_rows = w->pool_rows;
  bp.ws = wsl;
  bp.union_out = union_out;
  NSM_CHECK_CUDA(launch_pdl(union_build_kernel, 1, 1024, (size_t)NB * 4, s, bp));
  NSM_CHECK_CUDA(
      launch_pdl(union_x_kernel, kUnionRows, kUxThreads, 0, s, x, (int)x_dtype, (int)rows, (int)hidden, wsl));

  UnionMlpParams p{};
  p.gate = w->gate_packed;
  p.gate_am = w->gate_absmax;
  p.up = w->up_packed;
  p.up_am = w->up_absmax;
  p.gstride = w->gateup_block_stride ? w->gateup_block_stride : (int64_t)16 * hidden;
  p.gastride = w->gateup_absmax_block_stride ? w->gateup_absmax_block_stride : (int64_t)hidden / 2;
  p.down = w->down_packed;
  p.down_am = w->down_absmax;
  p.dbs = w->down_block_stride ? w->down_block_stride : (int64_t)16 * hidden;
  p.dabs = w->down_absmax_block_stride ? w->down_absmax_block_stride : (int64_t)hidden;
  p.gate_code = w->gate_code;
  p.up_code = w->up_code;
  p.down_code = w->down_code;
  p.H = hidden;
  p.rows = rows;
  p.ws = wsl;
  p.y = y;
  p.y_dtype = y_dtype;
  NSM_REQUIRE(p.gstride % 16 == 0 && (p.gastride * 4) % 16 == 0 && p.dbs % 16 == 0 && (p.dabs * 4) % 16 == 0,
              NSM_ERR_INVALID_ARG, "pool strides must be multiples of 16 bytes");
  const int gu_ctas = dev.sm_count * gu_per_sm;
  p.total_warps = gu_ctas * (kUnionThreads / 32);
  NSM_CHECK_CUDA(launch_pdl(union_gateup_kernel, gu_ctas, kUnionThreads, kSmemHead, s, p));
  NSM_CHECK_CUDA(launch_pdl(union_act_kernel, umax, 1024, 0, s, p));
  const int dn_ctas = dev.sm_count * dn_per_sm;
  NSM_CHECK_CUDA(launch_pdl(union_down_kernel, dn_ctas, kUdThreads, kUdSmem, s, p));
  NSM_CHECK_CUDA(launch_pdl(union_y_kernel, (hidden * kUnionRows + 255) / 256, 256, 0, s, p));
  if (union_count_out) NSM_CHECK_CUDA(cudaMemcpyAsync(union_count_out, wsl.u_count, sizeof(int32_t),
                                                      cudaMemcpyDeviceToDevice, s));
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

}  // extern "C"
