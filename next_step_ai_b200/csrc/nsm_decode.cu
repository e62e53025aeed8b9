// nsm_decode.cu -- single-token blockwise-sparse NF4 decode MLP for sm_100a.
//
// Pipeline of one decode step (one decoder layer, one token), all on one stream,
// chained with programmatic dependent launch:
//   1. router_latent_kernel   x prep (optional residual add of the previous
//                             layer's pending output + RMSNorm), fp16 x with
//                             per-64-column power-of-two scales, split-H
//                             partial latents x . enc_w^T.
//   2. router_scores_kernel   every CTA reduces the partial latents (norm scale,
//                             bias, basis top-k), then block scores
//                             clamp0(latent . score_w^T + b) (* down_block_norm).
//   3. router_topk_kernel     top-k (score desc, index asc) by radix select;
//                             compacts the selection into pool rows through
//                             the block map (resident table or shard range).
//   4. gateup_tma_kernel /    warps stream equal ranges of the (block, 64-column
//      gateup_kernel          tile) pairs: NF4 gather-GEMV of gate and up, fp32
//                             partials per block segment.
//   5. gateup_finalize_kernel fixed-order segment sums, SiLU(g)*u as fp16 with a
//                             per-block power-of-two scale.
//   6. down_tma_kernel /      warps stream equal ranges of the (row group,
//      down_kernel            block) pairs: NF4 column gather-GEMV, fp32
//                             partials per row-group segment.
//   7. down_finalize_kernel   fixed-order segment sums (+ bias) -> y; or, when
//                             the output is deferred, the next layer's router
//                             kernel sums the segments into the residual.
// Reference semantics: streaming_llama_runtime.py:4209-4238 (latent),
// :4311-4352 (scores/top-k), :5433-5492 (MLP math).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <string>

#include "nsm_common.cuh"
#include "nsm_internal.h"
#include "nsm_nf4.cuh"
#include "nsm_router.h"
#include "nsm_select.cuh"

namespace nsm {

// Identity rows 0..count-1 (gathered layouts).
__global__ void identity_rows_kernel(int* rows, int* count, int* sel, int n) {
  pdl_trigger();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    rows[i] = i;
    sel[i] = i;
  }
  // (row i of a gathered layout is block i of the gathered list)
  if (blockIdx.x == 0 && threadIdx.x == 0) *count = n;
}

// ============================================================================
// 3/4. NF4 gather-GEMV kernels: shared helpers
// ============================================================================
constexpr int kMlpThreads = 256;  // 8 warps per CTA, two CTAs per SM

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
  const __half* x16lo;  // remainder of x16 (the B operand's column 1)
  const float* xscale;
  const float* norm_scale;
  const void* act_mask;  // optional [U*32] (one row of flat_mask)
  int mask_dtype;
  float* gu_part;
  int* err;
  __half* act16;
  __half* act16lo;
  float* act_scale;
  float* act_out;  // optional fp32 [k][32]
  // fused_finalize != 0 (bulk-copy kernel only): the warp that completes a
  // block's units (counted on gu_ticket[s], zero between calls) applies
  // SiLU(gate)*up itself; no gateup_finalize_kernel follows
  int fused_finalize;
  unsigned* gu_ticket;
  int total_warps;
  int unit_tiles;  // tiles per stream unit (the partial segments follow the units)
  int max_rows;    // capacity of rows / partials (>= *count_ptr): prologues load this much without waiting for the count
  int wait_spins;  // bound of a warp's wait for its bulk copies (nsm_set_copy_wait_limit)
  // select != 0 (bulk-copy kernel only): the kernel selects the blocks itself
  // from the router's scores -- top `top_k` of NB, through the block map --
  // and CTA 0 writes rows_out / row_block_out / count_out for the later kernels
  int select;
  const float* scores;
  int NB, top_k;
  const int* slot_of_block;
  int block_begin, block_end, pool_rows;
  int* rows_out;
  int* row_block_out;
  int* count_out;
};

// One 64-column tile of one block, both projections: w[proj][rg] holds the
// lane's 8 bytes of row 16*rg+g (.x,.y) and of row 16*rg+g+8 (.z,.w);
// am[proj] holds the absmax of rows g, g+8, 16+g, 24+g.
struct GuTile {
  uint4 w[2][2];
  float4 am[2];
};

template <bool kTiled>
__device__ __forceinline__ void gu_load(const GateUpParams& p, const uint8_t* gb, const uint8_t* ub, const float* gab,
                                        const float* uab, int j, int lane, GuTile& r) {
  const int g = lane >> 2, t = lane & 3;
  if (kTiled) {
    const int64_t off = (int64_t)j * 1024 + lane * 16;
    r.w[0][0] = ldg_stream_u4(gb + off);
    r.w[0][1] = ldg_stream_u4(gb + off + 512);
    r.w[1][0] = ldg_stream_u4(ub + off);
    r.w[1][1] = ldg_stream_u4(ub + off + 512);
    r.am[0] = ldg_f4(gab + j * 32 + g * 4);
    r.am[1] = ldg_f4(uab + j * 32 + g * 4);
  } else {
    const int bpr = p.H >> 1, apr = p.H >> 6;
#pragma unroll
    for (int rg = 0; rg < 2; ++rg) {
      const int r0 = rg * 16 + g;
      const int64_t o0 = (int64_t)r0 * bpr + j * 32 + t * 8;
      const int64_t o1 = o0 + (int64_t)8 * bpr;
      const uint2 a0 = ldg_stream_u2(gb + o0), a1 = ldg_stream_u2(gb + o1);
      const uint2 c0 = ldg_stream_u2(ub + o0), c1 = ldg_stream_u2(ub + o1);
      r.w[0][rg] = make_uint4(a0.x, a0.y, a1.x, a1.y);
      r.w[1][rg] = make_uint4(c0.x, c0.y, c1.x, c1.y);
    }
    r.am[0] = make_float4(ldg_f32(gab + (int64_t)g * apr + j), ldg_f32(gab + (int64_t)(g + 8) * apr + j),
                          ldg_f32(gab + (int64_t)(g + 16) * apr + j), ldg_f32(gab + (int64_t)(g + 24) * apr + j));
    r.am[1] = make_float4(ldg_f32(uab + (int64_t)g * apr + j), ldg_f32(uab + (int64_t)(g + 8) * apr + j),
                          ldg_f32(uab + (int64_t)(g + 16) * apr + j), ldg_f32(uab + (int64_t)(g + 24) * apr + j));
  }
}

// 16 rows x 64 columns: four k=16 MMAs over the lane's bytes of two rows.
template <int kBase, int kTable>
__device__ __forceinline__ void gu_mma_rowgroup(uint32_t lb, const uint4 w, const uint32_t b[8], float d[4]) {
  mma_16816_z(d, lut_get<kBase>(w.x, lb, 0, kTable), lut_get<kBase>(w.z, lb, 0, kTable),
              lut_get<kBase>(w.x, lb, 1, kTable), lut_get<kBase>(w.z, lb, 1, kTable), b[0], b[1]);
  mma_16816(d, lut_get<kBase>(w.x, lb, 2, kTable), lut_get<kBase>(w.z, lb, 2, kTable),
            lut_get<kBase>(w.x, lb, 3, kTable), lut_get<kBase>(w.z, lb, 3, kTable), b[2], b[3]);
  mma_16816(d, lut_get<kBase>(w.y, lb, 0, kTable), lut_get<kBase>(w.w, lb, 0, kTable),
            lut_get<kBase>(w.y, lb, 1, kTable), lut_get<kBase>(w.w, lb, 1, kTable), b[4], b[5]);
  mma_16816(d, lut_get<kBase>(w.y, lb, 2, kTable), lut_get<kBase>(w.w, lb, 2, kTable),
            lut_get<kBase>(w.y, lb, 3, kTable), lut_get<kBase>(w.w, lb, 3, kTable), b[6], b[7]);
}

// Both projections of one tile: acc[proj][i] += (W_rows . x_tile) * absmax * xscale / alpha.
// The B operand carries x16 in column 0 (lanes g == 0) and x16lo in column 1
// (lanes g == 1), so D columns 0 + 1 (d[0] + d[1], d[2] + d[3] of lanes
// t == 0) hold the dot product with the hi + lo pair; xsg / xsu fold the
// tables' 1 / alpha into the tile's x scale.
template <int kBase, int kUpTable = 1>
__device__ __forceinline__ void gu_tile_mma(const GuTile& tile, const uint32_t b[8], float xsg, float xsu,
                                            uint32_t lb, float acc[2][4]) {
  float d[4];
#pragma unroll
  for (int rg = 0; rg < 2; ++rg) {
    gu_mma_rowgroup<kBase, 0>(lb, tile.w[0][rg], b, d);
    const float g0 = rg ? tile.am[0].z : tile.am[0].x, g1 = rg ? tile.am[0].w : tile.am[0].y;
    acc[0][rg * 2] = fmaf(d[0] + d[1], g0 * xsg, acc[0][rg * 2]);
    acc[0][rg * 2 + 1] = fmaf(d[2] + d[3], g1 * xsg, acc[0][rg * 2 + 1]);
    gu_mma_rowgroup<kBase, kUpTable>(lb, tile.w[1][rg], b, d);
    const float u0 = rg ? tile.am[1].z : tile.am[1].x, u1 = rg ? tile.am[1].w : tile.am[1].y;
    acc[1][rg * 2] = fmaf(d[0] + d[1], u0 * xsu, acc[1][rg * 2]);
    acc[1][rg * 2 + 1] = fmaf(d[2] + d[3], u1 * xsu, acc[1][rg * 2 + 1]);
  }
}

// xv: this lane's x vector -- x16 (or its shared-memory copy) for lanes
// g != 1, x16lo for lanes g == 1 (column 1 of the B operand).
template <int kBase, bool kStageX>
__device__ __forceinline__ void gu_compute(const GateUpParams& p, const GuTile& tile, int j, int t, uint32_t lb,
                                           const __half* xv, const float* xss, float ia0, float ia1,
                                           float acc[2][4]) {
  uint32_t b[8];
  float xs;
  const uint4 xa = kStageX ? *reinterpret_cast<const uint4*>(xv + j * 64 + t * 16) : ldg_u4(xv + j * 64 + t * 16);
  const uint4 xb =
      kStageX ? *reinterpret_cast<const uint4*>(xv + j * 64 + t * 16 + 8) : ldg_u4(xv + j * 64 + t * 16 + 8);
  b[0] = xa.x; b[1] = xa.y; b[2] = xa.z; b[3] = xa.w;
  b[4] = xb.x; b[5] = xb.y; b[6] = xb.z; b[7] = xb.w;
  xs = kStageX ? xss[j] : ldg_f32(p.xscale + j);
  gu_tile_mma<kBase>(tile, b, xs * ia0, xs * ia1, lb, acc);
}

constexpr int kStageRowsMax = 1024;  // pool rows staged in shared memory up to this count

struct GuPtrs {
  const uint8_t* g;
  const uint8_t* u;
  const float* ga;
  const float* ua;
};

__device__ __forceinline__ GuPtrs gu_ptrs(const GateUpParams& p, int prow) {
  return GuPtrs{p.gate + (int64_t)prow * p.gstride, p.up + (int64_t)prow * p.gstride,
                p.gate_am + (int64_t)prow * p.gastride, p.up_am + (int64_t)prow * p.gastride};
}

__device__ __forceinline__ void gu_flush(const GateUpParams& p, int s, int seg, int g, int t, float acc[2][4]) {
  // column 0 of the accumulator lives in lanes with t == 0
  if (t == 0) {
    float* part = p.gu_part + ((int64_t)s * kMaxUnitsPerSlot + seg) * 64;
#pragma unroll
    for (int pr = 0; pr < 2; ++pr)
#pragma unroll
      for (int i = 0; i < 4; ++i) part[pr * 32 + (i >> 1) * 16 + g + (i & 1) * 8] = acc[pr][i];
  }
#pragma unroll
  for (int pr = 0; pr < 2; ++pr)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[pr][i] = 0.f;
}

template <bool kTiled, bool kStageX, int kBase>
__device__ __forceinline__ void gateup_body(const GateUpParams& p, uint32_t lb, const __half* xs16, const float* xss,
                                            const int* rows, int count) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int tpr = p.H >> 6;
  const int total = count * tpr;
  const int nw = stream_warps(count, tpr, kMaxUnitsPerSlot, p.total_warps);
  if (warp_global >= nw) return;
  const int q0 = stream_begin(total, nw, warp_global), q1 = stream_begin(total, nw, warp_global + 1);
  int s = q0 / tpr, j = q0 - s * tpr;
  int seg = warp_global - stream_owner(total, nw, s * tpr);
  // lanes g == 1 read x16lo (from global memory: only x16 is staged)
  const __half* xv = g == 1 ? p.x16lo : (kStageX ? xs16 : p.x16);
  const float ia0 = lut_inv_alpha(0), ia1 = lut_inv_alpha(1);
  GuPtrs cp = gu_ptrs(p, rows[s]);
  GuTile ta, tb;
  gu_load<kTiled>(p, cp.g, cp.u, cp.ga, cp.ua, j, lane, ta);
  float acc[2][4] = {};
  int q = q0;
  // one pair: load the next pair into `nx`, compute `cur`, flush at a block
  // boundary or at the end of the range
  auto step = [&](GuTile& cur, GuTile& nx) -> bool {
    int sn = s, jn = j + 1;
    if (jn == tpr) { jn = 0; ++sn; }
    const bool more = q + 1 < q1;
    GuPtrs np = cp;
    if (more) {
      if (sn != s) np = gu_ptrs(p, rows[sn]);
      gu_load<kTiled>(p, np.g, np.u, np.ga, np.ua, jn, lane, nx);
    }
    gu_compute<kBase, kStageX>(p, cur, j, t, lb, xv, xss, ia0, ia1, acc);
    if (!more || sn != s) {
      gu_flush(p, s, seg, g, t, acc);
      seg = 0;  // this warp holds the first pair of the next block
    }
    s = sn;
    j = jn;
    cp = np;
    ++q;
    return more;
  };
  while (true) {
    if (!step(ta, tb)) break;
    if (!step(tb, ta)) break;
  }
}

// RMSNorm scale, biases, mask and SiLU(gate)*up of neuron `lane` of pool row
// s from its summed gate/up dot products; fp16 with a per-block power-of-two
// scale (the whole warp calls this for one block).
__device__ __forceinline__ void gu_finalize_apply(const GateUpParams& p, int s, int lane, float gsum, float usum,
                                                  float ns) {
  gsum *= ns;
  usum *= ns;
  if (p.gate_bias != nullptr || p.up_bias != nullptr) {
    const int bi = (p.bias_by_block ? __ldcg(p.row_block + s) : s) * 32 + lane;
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
  const float v = act * (1.f / sc);
  const __half h = __float2half_rn(v);
  p.act16[(int64_t)s * 32 + lane] = h;
  p.act16lo[(int64_t)s * 32 + lane] = __float2half_rn(v - __half2float(h));
  if (lane == 0) p.act_scale[s] = sc;
}

// One CTA (256 threads) per block: thread (q, lane) sums the column-range
// partials q, q+8, ... of neuron `lane` (gate and up), the 8 sums combine in
// fixed order, then RMSNorm scale, biases, mask and SiLU(gate)*up are applied
// and written as fp16 with a per-block power-of-two scale.
__global__ void __launch_bounds__(256) gateup_finalize_kernel(GateUpParams p) {
  __shared__ float red[2][8][32];
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, q0 = threadIdx.x >> 5;
  const int s = blockIdx.x;
  // segments q0, q0+8, q0+16, q0+24 go out with the count (one round trip;
  // the ones past this block's segment count are ignored)
  const int count = *p.count_ptr;
  const float* base = p.gu_part + (int64_t)s * kMaxUnitsPerSlot * 64;
  float vg[4], vu[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    vg[u] = ldcg_f32(base + (q0 + 8 * u) * 64 + lane);
    vu[u] = ldcg_f32(base + (q0 + 8 * u) * 64 + 32 + lane);
  }
  const float ns = p.norm_scale ? ldcg_f32(p.norm_scale) : 1.f;
  if (s >= count) return;
  const int cps = (p.H >> 6) / p.unit_tiles;
  const int nw = stream_warps(count, cps, kMaxUnitsPerSlot, p.total_warps);
  const int ups = stream_owner(count * cps, nw, s * cps + cps - 1) - stream_owner(count * cps, nw, s * cps) + 1;
  float gsum = 0.f, usum = 0.f;
#pragma unroll
  for (int u = 0; u < 4; ++u)
    if (q0 + 8 * u < ups) {
      gsum += vg[u];
      usum += vu[u];
    }
  for (int q = q0 + 32; q < ups; q += 8) {
    gsum += ldcg_f32(base + q * 64 + lane);
    usum += ldcg_f32(base + q * 64 + 32 + lane);
  }
  red[0][q0][lane] = gsum;
  red[1][q0][lane] = usum;
  __syncthreads();
  if (q0 != 0) return;
  gsum = 0.f;
  usum = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    gsum += red[0][q][lane];
    usum += red[1][q][lane];
  }
  gu_finalize_apply(p, s, lane, gsum, usum, ns);
}

constexpr int kStageXMaxHidden = 16384;

template <bool kTiled, bool kStageX>
__global__ void __launch_bounds__(kMlpThreads, 2) gateup_kernel(GateUpParams p) {
  pdl_trigger();
  build_lut_alpha(p.gate_code, p.up_code);
  pdl_wait();  // rows, count, x16 come from the router kernels
  __half* xs16 = reinterpret_cast<__half*>(reinterpret_cast<char*>(g_lut_smem) + kSmemHead);
  float* xss = reinterpret_cast<float*>(xs16 + (kStageX ? p.H : 0));
  int* srows = reinterpret_cast<int*>(xss + (kStageX ? p.H / 64 : 0));
  const int count = *p.count_ptr;
  if (kStageX) {
    const uint4* src = reinterpret_cast<const uint4*>(p.x16);
    uint4* dst = reinterpret_cast<uint4*>(xs16);
    for (int i = threadIdx.x; i < p.H / 8; i += blockDim.x) dst[i] = __ldcg(src + i);
    for (int i = threadIdx.x; i < p.H / 64; i += blockDim.x) xss[i] = __ldcg(p.xscale + i);
  }
  const bool stage_rows = count <= kStageRowsMax;
  if (stage_rows)
    for (int i = threadIdx.x; i < count; i += blockDim.x) srows[i] = __ldcg(p.rows + i);
  __syncthreads();
  const int* rows = stage_rows ? srows : p.rows;
  const uint32_t lb = (threadIdx.x & 31) * 4u;
  const uint32_t base = lut_base_addr();
  if (base == 0x400u)
    gateup_body<kTiled, kStageX, 0x400>(p, lb, xs16, xss, rows, count);
  else
    gateup_body<kTiled, kStageX, -1>(p, lb, xs16, xss, rows, count);
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
  const __half* act16lo;  // remainder of act16 (the B operand's column 1)
  const float* act_scale;
  float* ypart;
  int* err;
  int group_log2;  // log2 of the rows per down reduction group (5 or 6)
  int* meta;       // ws.down_meta: the launch records total_warps and group_log2 there
  void* y;
  int y_dtype;
  int total_warps;
  int max_rows;  // capacity of rows / act16 (>= *count_ptr): the prologue loads this much without waiting for the count
  int wait_spins;  // bound of a warp's wait for its bulk copies (nsm_set_copy_wait_limit)
};

__device__ __forceinline__ void record_down_meta(const DownParams& p) {
  if (blockIdx.x == 0 && threadIdx.x == 0 && p.meta != nullptr) {
    p.meta[0] = p.total_warps;
    p.meta[1] = p.group_log2;
  }
}

constexpr int kDownBatch = 4;          // blocks per load batch (two batches in flight)
constexpr int kStageActMaxSlots = 256;  // act16 + scale + row staged in shared memory up to this k

template <bool kTiled>
__device__ __forceinline__ void down_load(const DownParams& p, int prow, int rt, int lane, uint4& w, float4& am) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* base = p.down + (int64_t)prow * p.dbs;
  const float* abase = p.down_am + (int64_t)(p.pair ? (prow >> 1) : prow) * p.dabs;
  if (kTiled) {
    w = ldg_stream_u4(base + (int64_t)rt * 512 + lane * 16);
    am = ldg_f4(abase + rt * 32 + g * 4);
  } else {
    const int r0 = rt * 32 + g;
    w.x = ldg_u32(base + (int64_t)r0 * p.drs + t * 4);
    w.y = ldg_u32(base + (int64_t)(r0 + 8) * p.drs + t * 4);
    w.z = ldg_u32(base + (int64_t)(r0 + 16) * p.drs + t * 4);
    w.w = ldg_u32(base + (int64_t)(r0 + 24) * p.drs + t * 4);
    am.x = ldg_f32(abase + (int64_t)r0 * p.dars);
    am.y = ldg_f32(abase + (int64_t)(r0 + 8) * p.dars);
    am.z = ldg_f32(abase + (int64_t)(r0 + 16) * p.dars);
    am.w = ldg_f32(abase + (int64_t)(r0 + 24) * p.dars);
  }
}

template <int kBase>
__device__ __forceinline__ void down_mma(uint32_t lb, uint32_t w0, uint32_t w1, const uint4 bf, float d[4]) {
  mma_16816_z(d, lut_get<kBase>(w0, lb, 0, 0), lut_get<kBase>(w1, lb, 0, 0), lut_get<kBase>(w0, lb, 1, 0),
              lut_get<kBase>(w1, lb, 1, 0), bf.x, bf.y);
  mma_16816(d, lut_get<kBase>(w0, lb, 2, 0), lut_get<kBase>(w1, lb, 2, 0), lut_get<kBase>(w0, lb, 3, 0),
            lut_get<kBase>(w1, lb, 3, 0), bf.z, bf.w);
}

struct DownBatch {
  uint4 w[kDownBatch];
  float4 am[kDownBatch];
};

// Down pairs are (32-row tile rt, slot s), rt-major: pair q = rt * count + s.
__device__ __forceinline__ int down_stream_warps(int count, int RT, int total_warps) {
  return stream_warps(RT, count, kMaxSlotGroups, total_warps);
}

// The B operand carries act16 in column 0 (lanes g == 0) and act16lo in
// column 1 (lanes g == 1); D columns 0 + 1 hold the dot product with the pair.
template <bool kTiled, bool kStage, int kBase>
__device__ __forceinline__ void down_body(const DownParams& p, uint32_t lb, const __half* sact,
                                          const __half* sactlo, const float* sscale, const int* rows, int count) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const __half* av = g == 1 ? (kStage ? sactlo : p.act16lo) : (kStage ? sact : p.act16);
  const float ia = lut_inv_alpha(0);
  const int warp_global = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int RT = p.H >> 5;
  const int total = RT * count;
  const int nw = down_stream_warps(count, RT, p.total_warps);
  if (warp_global >= nw) return;
  const int q0 = stream_begin(total, nw, warp_global), q1 = stream_begin(total, nw, warp_global + 1);
  int rt = q0 / count, s = q0 - rt * count;  // compute cursor
  int seg = warp_global - stream_owner(total, nw, rt * count);
  int lrt = rt, ls = s;                      // load cursor
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // rows g, g+8, 16+g, 24+g of tile rt
  DownBatch b0, b1;
  auto load_batch = [&](int qb, DownBatch& b) {
#pragma unroll
    for (int i = 0; i < kDownBatch; ++i) {
      if (qb + i < q1) {
        down_load<kTiled>(p, rows[ls], lrt, lane, b.w[i], b.am[i]);
        if (++ls == count) { ls = 0; ++lrt; }
      }
    }
  };
  auto compute_batch = [&](int qb, const DownBatch& b) {
#pragma unroll
    for (int i = 0; i < kDownBatch; ++i) {
      const int q = qb + i;
      if (q < q1) {
        uint4 bf;
        float as;
        if (kStage) {
          bf = *reinterpret_cast<const uint4*>(av + s * 32 + t * 8);
          as = sscale[s] * ia;
        } else {
          bf = ldg_u4(av + (int64_t)s * 32 + t * 8);
          as = ldg_f32(p.act_scale + s) * ia;
        }
        float d[4];
        down_mma<kBase>(lb, b.w[i].x, b.w[i].y, bf, d);
        acc[0] = fmaf(d[0] + d[1], b.am[i].x * as, acc[0]);
        acc[1] = fmaf(d[2] + d[3], b.am[i].y * as, acc[1]);
        down_mma<kBase>(lb, b.w[i].z, b.w[i].w, bf, d);
        acc[2] = fmaf(d[0] + d[1], b.am[i].z * as, acc[2]);
        acc[3] = fmaf(d[2] + d[3], b.am[i].w * as, acc[3]);
        if (++s == count || q + 1 == q1) {
          if (t == 0) {
            float* yp = p.ypart + (int64_t)seg * p.H + rt * 32;
#pragma unroll
            for (int r = 0; r < 4; ++r) yp[(r >> 1) * 16 + g + (r & 1) * 8] = acc[r];
          }
          acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
          seg = 0;  // this warp holds the first pair of the next row tile
          if (s == count) { s = 0; ++rt; }
        }
      }
    }
  };
  load_batch(q0, b0);
  for (int qb = q0; qb < q1; qb += 2 * kDownBatch) {
    if (qb + kDownBatch < q1) load_batch(qb + kDownBatch, b1);
    compute_batch(qb, b0);
    if (qb + kDownBatch >= q1) break;
    if (qb + 2 * kDownBatch < q1) load_batch(qb + 2 * kDownBatch, b0);
    compute_batch(qb + kDownBatch, b1);
  }
}

// Four threads per output row: each sums every fourth block-group partial,
// the four sums combine in fixed order.
__global__ void __launch_bounds__(256) down_finalize_kernel(DownParams p) {
  pdl_trigger();
  pdl_wait();
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = gtid >> 2, q0 = gtid & 3;
  const int count = *p.count_ptr;
  float y = 0.f;
  if (h < p.H && count > 0) {
    // reduction groups: 32-row tiles (register kernel) or 64-row groups (bulk-copy kernel)
    const int RT = p.H >> p.group_log2, rt = h >> p.group_log2;
    const int nw = stream_warps(RT, count, kMaxSlotGroups, p.total_warps);
    const int sg = stream_owner(RT * count, nw, rt * count + count - 1) - stream_owner(RT * count, nw, rt * count) + 1;
#pragma unroll 4
    for (int q = q0; q < sg; q += 4) y += ldcg_f32(p.ypart + (int64_t)q * p.H + h);
  }
  const float y1 = __shfl_down_sync(0xffffffffu, y, 1);
  const float y2 = __shfl_down_sync(0xffffffffu, y, 2);
  const float y3 = __shfl_down_sync(0xffffffffu, y, 3);
  if (h >= p.H || q0 != 0) return;
  y = (y + y1) + (y2 + y3);
  if (p.down_bias) y += load_as_f32(p.down_bias, p.bias_dtype, h);
  store_from_f32(p.y, p.y_dtype, h, y);
}

template <bool kTiled, bool kStage>
__global__ void __launch_bounds__(kMlpThreads, 2) down_kernel(DownParams p) {
  pdl_trigger();
  build_lut_alpha(p.down_code, p.down_code, false);  // the down loops read table 0 only
  pdl_wait();  // act16 / act_scale come from the gate/up kernel
  record_down_meta(p);
  const int count = *p.count_ptr;
  __half* sact = reinterpret_cast<__half*>(reinterpret_cast<char*>(g_lut_smem) + kSmemHead);
  float* sscale = reinterpret_cast<float*>(sact + kStageActMaxSlots * 32);
  int* srows = reinterpret_cast<int*>(sscale + kStageActMaxSlots);
  __half* sactlo = reinterpret_cast<__half*>(srows + kStageActMaxSlots);
  if (kStage) {
    const uint4* src = reinterpret_cast<const uint4*>(p.act16);
    const uint4* srclo = reinterpret_cast<const uint4*>(p.act16lo);
    uint4* dst = reinterpret_cast<uint4*>(sact);
    uint4* dstlo = reinterpret_cast<uint4*>(sactlo);
    for (int i = threadIdx.x; i < count * 4; i += blockDim.x) {
      dst[i] = __ldcg(src + i);
      dstlo[i] = __ldcg(srclo + i);
    }
    for (int i = threadIdx.x; i < count; i += blockDim.x) {
      sscale[i] = __ldcg(p.act_scale + i);
      srows[i] = __ldcg(p.rows + i);
    }
  }
  __syncthreads();
  const int* rows = kStage ? srows : p.rows;
  const uint32_t lb = (threadIdx.x & 31) * 4u;
  const uint32_t base = lut_base_addr();
  if (base == 0x400u)
    down_body<kTiled, kStage, 0x400>(p, lb, sact, sactlo, sscale, rows, count);
  else
    down_body<kTiled, kStage, -1>(p, lb, sact, sactlo, sscale, rows, count);
}

// ============================================================================
// 4b/6b. bulk-copy pipelined variants for the tiled pool layouts
// ============================================================================
// One CTA of kTmaWarps warps per SM.  Each warp owns a ring of shared-memory
// stages that its lane 0 fills with cp.async.bulk (one copy per contiguous
// tiled run: a 1 KB gate/up tile, a 512 B down row tile, their absmax), so a
// warp keeps kStages tiles in flight without holding them in registers.  A
// stage is refilled only after the warp's MMAs consumed the registers read
// from it.  Waits are bounded; a wait that runs out records NSM_ERR_TIMEOUT in
// the workspace error word, waits (bounded) for the warp's copies still in
// flight and stops the warp.
#ifndef NSM_TMA_WARPS
#define NSM_TMA_WARPS 16
#endif
#ifndef NSM_GU_STAGES
#define NSM_GU_STAGES 2
#endif
#ifndef NSM_GU_UNIT_TILES
#define NSM_GU_UNIT_TILES 2
#endif
#ifndef NSM_DN_STAGES
#define NSM_DN_STAGES 3
#endif
constexpr int kTmaWarps = NSM_TMA_WARPS;
constexpr int kTmaThreads = kTmaWarps * 32;
#ifndef NSM_GU_WARPS
#define NSM_GU_WARPS 10
#endif
constexpr int kGuWarps = NSM_GU_WARPS;  // gate/up: fewer warps, two-tile stages
constexpr int kGuThreads = kGuWarps * 32;
constexpr int kGuStages = NSM_GU_STAGES;
constexpr int kGuUnitTiles = NSM_GU_UNIT_TILES;
constexpr int kGuStageBytes = kGuUnitTiles * (2048 + 256);  // gate tiles, up tiles, gate absmax, up absmax
constexpr int kDnStages = NSM_DN_STAGES;
#ifndef NSM_DN_PAIRS_PER_STAGE
#define NSM_DN_PAIRS_PER_STAGE 2
#endif
constexpr int kDnPairsPerStage = NSM_DN_PAIRS_PER_STAGE;
constexpr int kDnStageBytes = kDnPairsPerStage * (1024 + 256);
// shared-memory layout (bytes from the dynamic base)
constexpr int kGuX16Off = kSmemHead;
// x16lo sits 16 bytes past a bank-aligned start: the lanes reading it (g == 1)
// then hit the four banks the x16 lanes of the same t leave free
constexpr int kGuX16LoOff = kGuX16Off + kStageXMaxHidden * 2 + 16;
constexpr int kGuXsOff = kGuX16Off + 2 * kStageXMaxHidden * 2 + 128;
constexpr int kGuRowsOff = kGuXsOff + (kStageXMaxHidden / 64) * 4;
constexpr int kGuRingOff = kGuRowsOff + kStageRowsMax * 4;
constexpr int kGuBarOff = kGuRingOff + kGuWarps * kGuStages * kGuStageBytes;
constexpr int kGuTmaSmem = kGuBarOff + (kGuWarps * kGuStages + 1) * 8;  // + the x staging barrier
constexpr int kDnActOff = kSmemHead;
// act16lo sits 64 bytes past a bank-aligned start: the lanes reading it (g == 1)
// then hit the 16 banks the act16 lanes leave free
constexpr int kDnActLoOff = kDnActOff + kStageActMaxSlots * 64 + 64;
constexpr int kDnScaleOff = kDnActOff + 2 * kStageActMaxSlots * 64 + 128;
constexpr int kDnRowsOff = kDnScaleOff + kStageActMaxSlots * 4;
constexpr int kDnRingOff = kDnRowsOff + kStageActMaxSlots * 4;
constexpr int kDnBarOff = kDnRingOff + kTmaWarps * kDnStages * kDnStageBytes;
constexpr int kDnTmaSmem = kDnBarOff + (kTmaWarps * kDnStages + 1) * 8;  // + the act staging barrier
// Shared-codebook variant (gate and up codebooks equal, NSM_LAYOUT_SHARED_CODE):
// one lookup table serves both projections, so the second table's half of
// every 256-byte entry is free and holds x16lo (tile j's 128 bytes in entry
// j, rotated by 16 bytes so its lanes use the banks the x16 lanes leave
// free); the 32 KB saved go to two more warps.
constexpr int kGu1Warps = 12;
constexpr int kGu1Threads = kGu1Warps * 32;
constexpr int kGu1XsOff = kGuX16Off + kStageXMaxHidden * 2;
constexpr int kGu1RowsOff = kGu1XsOff + (kStageXMaxHidden / 64) * 4;
constexpr int kGu1RingOff = kGu1RowsOff + kStageRowsMax * 4;
constexpr int kGu1BarOff = kGu1RingOff + kGu1Warps * kGuStages * kGuStageBytes;
constexpr int kGu1TmaSmem = kGu1BarOff + (kGu1Warps * kGuStages + 1) * 8;
static_assert(kGu1TmaSmem <= 227 * 1024, "gate/up ring (shared codebook) does not fit in shared memory");
static_assert(kGu1RingOff % 128 == 0, "rings must be 128-byte aligned");
// x16lo's staging in the ring (shared codebook), past the selection's scratch
constexpr int kGu1XloStageOff = 40 * 1024;
static_assert(kGu1XloStageOff + kStageXMaxHidden * 2 <= kGu1Warps * kGuStages * kGuStageBytes,
              "x16lo staging must fit in the gate/up ring");
static_assert(kStageXMaxHidden / 64 <= 256, "x16lo needs one lookup entry per 64-column tile");
template <bool kOne> struct GuCfg {
  static constexpr int kWarps = kOne ? kGu1Warps : kGuWarps;
  static constexpr int kXsOff = kOne ? kGu1XsOff : kGuXsOff;
  static constexpr int kRowsOff = kOne ? kGu1RowsOff : kGuRowsOff;
  static constexpr int kRingOff = kOne ? kGu1RingOff : kGuRingOff;
  static constexpr int kBarOff = kOne ? kGu1BarOff : kGuBarOff;
};
// byte offset of x16lo's 16-byte chunk c (0..7) of tile j inside the lookup table
__host__ __device__ constexpr uint32_t gu1_xlo_off(int j, int c) {
  return (uint32_t)j * 256u + 128u + (uint32_t)((c * 16 + 16) & 127);
}
static_assert(kGuTmaSmem <= 227 * 1024, "gate/up ring does not fit in shared memory");
static_assert(kDnTmaSmem <= 227 * 1024, "down ring does not fit in shared memory");
static_assert(kGuRingOff % 128 == 0 && kDnRingOff % 128 == 0, "rings must be 128-byte aligned");

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// After a failed wait: bounded waits for the batches [consumed, issued) that a
// warp's ring may still be receiving (batch b sits in stage b % kStages and
// completes phase (b / kStages) & 1 of that stage's mbarrier).
template <int kStages>
__device__ __forceinline__ void drain_ring(uint32_t wbar, int consumed, int issued) {
  for (int b = consumed; b < issued; ++b) mbar_wait(wbar + 8u * (uint32_t)(b % kStages), (uint32_t)((b / kStages) & 1));
}

// Counts a flushed segment of `units` units of block s on its ticket; true
// for the warp whose segment completed the block (it then owes the block's
// SiLU(gate)*up, gu_finalize_block).  The partial stores of lanes t == 0 are
// made visible before the count.
__device__ __forceinline__ bool gu_ticket_add(const GateUpParams& p, int s, int units, int cps, int lane) {
  __threadfence();
  __syncwarp();
  unsigned old = 0u;
  if (lane == 0) old = atomicAdd(p.gu_ticket + s, (unsigned)units);
  old = __shfl_sync(0xffffffffu, old, 0);
  return old + (unsigned)units == (unsigned)cps;
}

// gateup_finalize_kernel's work for block s by one warp (lane = neuron), in the
// same summation order: segment q goes to group q mod 8, each group sums its
// segments in order, the 8 group sums combine in order.  Then the ticket is
// reset for the next call.  Split in two so that a warp owing several blocks
// has all their partial loads in flight at once (gu_finalize_load for each,
// then gu_finalize_store for each).
__device__ __forceinline__ void gu_finalize_load(const GateUpParams& p, int s, int cps, int total, int nw, int lane,
                                                 float (&vg)[8], float (&vu)[8]) {
  const int ups = stream_owner(total, nw, s * cps + cps - 1) - stream_owner(total, nw, s * cps) + 1;
  const float* base = p.gu_part + (int64_t)s * kMaxUnitsPerSlot * 64;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    vg[q] = q < ups ? ldcg_f32(base + q * 64 + lane) : 0.f;
    vu[q] = q < ups ? ldcg_f32(base + q * 64 + 32 + lane) : 0.f;
  }
  for (int q0 = 8; q0 < ups; q0 += 8) {
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (q0 + u < ups) {
        vg[u] += ldcg_f32(base + (q0 + u) * 64 + lane);
        vu[u] += ldcg_f32(base + (q0 + u) * 64 + 32 + lane);
      }
  }
}
__device__ __forceinline__ void gu_finalize_store(const GateUpParams& p, int s, int lane, const float (&vg)[8],
                                                  const float (&vu)[8], float ns) {
  float gsum = 0.f, usum = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    gsum += vg[q];
    usum += vu[q];
  }
  gu_finalize_apply(p, s, lane, gsum, usum, ns);
  __syncwarp();
  if (lane == 0) p.gu_ticket[s] = 0u;
}
__device__ __forceinline__ void gu_finalize_block(const GateUpParams& p, int s, int cps, int total, int nw,
                                                  int lane) {
  __threadfence();
  float vg[8], vu[8];
  gu_finalize_load(p, s, cps, total, nw, lane, vg, vu);
  gu_finalize_store(p, s, lane, vg, vu, p.norm_scale ? ldcg_f32(p.norm_scale) : 1.f);
}

// A ring stage holds one *unit* of kGuUnitTiles adjacent tiles of one block
// (gate kGuUnitTiles KB, up kGuUnitTiles KB, their absmax runs): four bulk
// copies and one round of cursor bookkeeping per unit instead of per tile.
template <int kBase, bool kOne>
__device__ __forceinline__ void gateup_tma_body(const GateUpParams& p, uint32_t lb, uint32_t xhi_s, uint32_t xlo_s,
                                                uint32_t xss_s, const int* rows, int count, uint32_t ring,
                                                uint32_t bar0) {
  constexpr int UT = kGuUnitTiles;
  constexpr int kUpTable = kOne ? 0 : 1;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  // B operand column 0 (lanes g == 0) is x16, column 1 (lanes g == 1) x16lo:
  // tile jj's fragment of this lane at xbase + jj * xstride + xoff0 / xoff1
  const bool lo = g == 1;
  const uint32_t xbase = lo ? xlo_s : xhi_s;
  const uint32_t xstride = (kOne && lo) ? 256u : 128u;
  const uint32_t xoff0 = (kOne && lo) ? gu1_xlo_off(0, 2 * t) : (uint32_t)(t * 32);
  const uint32_t xoff1 = (kOne && lo) ? gu1_xlo_off(0, 2 * t + 1) : (uint32_t)(t * 32 + 16);
  const float ia0 = lut_inv_alpha(0), ia1 = lut_inv_alpha(kUpTable);
  const int warp = threadIdx.x >> 5;
  const int warp_global = blockIdx.x * GuCfg<kOne>::kWarps + warp;
  const int cps = (p.H >> 6) / UT;  // units per block
  const int total = count * cps;
  const int nw = stream_warps(count, cps, kMaxUnitsPerSlot, p.total_warps);
  if (warp_global >= nw) return;
  const int q0 = stream_begin(total, nw, warp_global), q1 = stream_begin(total, nw, warp_global + 1);
  const uint32_t wring = ring + (uint32_t)(warp * kGuStages * kGuStageBytes);
  const uint32_t wbar = bar0 + (uint32_t)(warp * kGuStages * 8);
  const uint64_t pol = l2_evict_first_policy();
  // load cursor: source pointers of the next unit to fetch
  int ls = q0 / cps, lj = q0 - ls * cps;
  const uint8_t* lg;
  const uint8_t* lu;
  const float* lga;
  const float* lua;
  auto load_slot = [&]() {
    const int prow = rows[ls];
    lg = p.gate + (int64_t)prow * p.gstride + (int64_t)lj * (UT * 1024);
    lu = p.up + (int64_t)prow * p.gstride + (int64_t)lj * (UT * 1024);
    lga = p.gate_am + (int64_t)prow * p.gastride + lj * (UT * 32);
    lua = p.up_am + (int64_t)prow * p.gastride + lj * (UT * 32);
  };
  int issued = 0;
  auto issue_next = [&](int stage) {  // fetch the cursor's unit into `stage`, advance the cursor
    ++issued;
    if (lane == 0) {
      fence_proxy_async_smem();  // the warp's reads of this stage come first
      const uint32_t dst = wring + (uint32_t)(stage * kGuStageBytes);
      const uint32_t bar = wbar + 8u * (uint32_t)stage;
      mbar_arrive_expect_tx(bar, kGuStageBytes);
      bulk_g2s(dst, lg, UT * 1024u, bar, pol);
      bulk_g2s(dst + UT * 1024, lu, UT * 1024u, bar, pol);
      bulk_g2s(dst + UT * 2048, lga, UT * 128u, bar, pol);
      bulk_g2s(dst + UT * 2048 + UT * 128, lua, UT * 128u, bar, pol);
    }
    lg += UT * 1024;
    lu += UT * 1024;
    lga += UT * 32;
    lua += UT * 32;
    if (++lj == cps) {
      lj = 0;
      if (++ls < count) load_slot();
    }
  };
  load_slot();
#pragma unroll
  for (int i = 0; i < kGuStages; ++i)
    if (q0 + i < q1) issue_next(i);

  int s = q0 / cps, j = q0 - s * cps;  // unit j of block s
  int seg = warp_global - stream_owner(total, nw, s * cps);
  const int s_first = s;
  int j_seg = j;                    // the unit the current segment started at
  unsigned long long owed = 0ull;   // bit s - s_first: this warp finalizes block s
  uint32_t xa = xbase + (uint32_t)(j * UT) * xstride;  // the unit's first tile
  uint32_t xsa = xss_s + (uint32_t)(j * UT * 4);
  float acc[2][4] = {};
  uint32_t phase = 0;
  int q = q0;
  bool ok = true;
  while (q < q1 && ok) {
#pragma unroll
    for (int st = 0; st < kGuStages; ++st) {
      if (q < q1 && ok) {
        const uint32_t bar = wbar + 8u * st;
        if (!mbar_wait(bar, phase, p.wait_spins)) {
          ok = false;
        } else {
          const uint32_t sb = wring + (uint32_t)(st * kGuStageBytes);
#pragma unroll
          for (int tt = 0; tt < UT; ++tt) {
            GuTile tile;
            tile.w[0][0] = lds_u4(sb + tt * 1024 + lane * 16);
            tile.w[0][1] = lds_u4(sb + tt * 1024 + 512 + lane * 16);
            tile.w[1][0] = lds_u4(sb + UT * 1024 + tt * 1024 + lane * 16);
            tile.w[1][1] = lds_u4(sb + UT * 1024 + tt * 1024 + 512 + lane * 16);
            tile.am[0] = lds_f4(sb + UT * 2048 + tt * 128 + g * 16);
            tile.am[1] = lds_f4(sb + UT * 2048 + UT * 128 + tt * 128 + g * 16);
            const uint4 x0 = lds_u4(xa + tt * xstride + xoff0), x1 = lds_u4(xa + tt * xstride + xoff1);
            const uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            float xs;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(xs) : "r"(xsa + tt * 4));
            gu_tile_mma<kBase, kUpTable>(tile, bx, xs * ia0, xs * ia1, lb, acc);
          }
          __syncwarp();
          if (q + kGuStages < q1) issue_next(st);
          ++q;
          xa += UT * xstride;
          xsa += UT * 4;
          if (++j == cps || q == q1) {
            gu_flush(p, s, seg, g, t, acc);
            if (p.fused_finalize && gu_ticket_add(p, s, j - j_seg, cps, lane)) {
              // a warp's range covers a few blocks; past 64 it finalizes at once
              if (s - s_first < 64) owed |= 1ull << (s - s_first);
              else gu_finalize_block(p, s, cps, total, nw, lane);
            }
            seg = 0;  // this warp holds the first unit of the next block
            j_seg = j;
            if (j == cps) {
              j = 0;
              j_seg = 0;
              ++s;
              xa = xbase;
              xsa = xss_s;
            }
          }
        }
      }
    }
    phase ^= 1u;
  }
  if (!ok) {
    record_error(p.err, NSM_ERR_TIMEOUT);
    drain_ring<kGuStages>(wbar, q - q0, issued);
    return;
  }
  // SiLU(gate)*up of the blocks whose last units this warp counted, two at a
  // time with both blocks' partial loads in flight together
  if (owed) {
    __threadfence();
    const float ns = p.norm_scale ? ldcg_f32(p.norm_scale) : 1.f;
    while (owed) {
      const int b0 = __ffsll((long long)owed) - 1;
      owed &= owed - 1ull;
      const int b1 = owed ? __ffsll((long long)owed) - 1 : -1;
      if (b1 >= 0) owed &= owed - 1ull;
      float vg0[8], vu0[8], vg1[8], vu1[8];
      gu_finalize_load(p, s_first + b0, cps, total, nw, lane, vg0, vu0);
      if (b1 >= 0) gu_finalize_load(p, s_first + b1, cps, total, nw, lane, vg1, vu1);
      gu_finalize_store(p, s_first + b0, lane, vg0, vu0, ns);
      if (b1 >= 0) gu_finalize_store(p, s_first + b1, lane, vg1, vu1, ns);
    }
  }
}

// Block map of the fused selection (the router kernels' map_block).
__device__ __forceinline__ int gu_map_block(const GateUpParams& p, int b) {
  int r;
  if (p.slot_of_block != nullptr) r = __ldg(p.slot_of_block + b);
  else r = (b >= p.block_begin && b < p.block_end) ? b - p.block_begin : -1;
  return (r >= 0 && r < p.pool_rows) ? r : -1;
}

// The decode path's block selection inside the gate/up kernel (every CTA, the
// same result): the router's scores -> order-preserving keys in `keys`, exact
// top-k (ties at the threshold to the lower block id), the selected blocks
// present in this pool compacted in block-id order into srows.  CTA 0 also
// writes the rows, their block ids and the count for the later kernels.
// Returns the count.  Everything lives in dynamic shared memory.
__device__ __forceinline__ int gu_select_blocks(const GateUpParams& p, uint32_t* keys, RadixSelectSmem& S, int* srows) {
  const int tid = threadIdx.x, NB = p.NB;
  uint32_t kor = 0u, kand = 0xffffffffu;
  for (int i0 = 0; i0 < NB; i0 += 8 * (int)blockDim.x) {
    float v[8];  // 8 score loads in flight per thread
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * (int)blockDim.x + tid;
      v[u] = i < NB ? ldcg_f32(p.scores + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * (int)blockDim.x + tid;
      if (i < NB) {
        const uint32_t key = orderable(v[u]);
        keys[i] = key;
        kor |= key;
        kand &= key;
      }
    }
  }
  block_radix_select(keys, NB, p.top_k, kor, kand, S);
  const uint32_t thr = S.prefix;
  const int take_eq = S.need;
  const bool split = take_eq != S.bin_count;  // a tie at the threshold is split: rank the equal keys
  const int per = (NB + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = min(NB, tid * per), hi = min(NB, lo + per);  // contiguous chunk: block-id order
  int tot, eq_before = 0;
  if (split) {
    int n_eq = 0;
    for (int i = lo; i < hi; ++i) n_eq += keys[i] == thr;
    eq_before = block_exclusive_scan_s(n_eq, &tot, S.wsum);
  }
  int m = 0;
  for (int i = lo, e = eq_before; i < hi; ++i) {
    const uint32_t key = keys[i];
    const bool sel = key > thr || (key == thr && (!split || e++ < take_eq));
    m += sel && gu_map_block(p, i) >= 0;
  }
  int pos = block_exclusive_scan_s(m, &tot, S.wsum);
  for (int i = lo, e = eq_before; i < hi; ++i) {
    const uint32_t key = keys[i];
    const bool sel = key > thr || (key == thr && (!split || e++ < take_eq));
    const int r = sel ? gu_map_block(p, i) : -1;
    if (r < 0) continue;
    srows[pos] = r;
    if (blockIdx.x == 0) {
      p.rows_out[pos] = r;
      p.row_block_out[pos] = i;
    }
    ++pos;
  }
  if (blockIdx.x == 0 && tid == 0) *p.count_out = tot;
  return tot;
}
// The same selection with the keys in registers (NB <= kSelKeysPerThread *
// blockDim), in two steps so that the score loads leave first:
// gu_select_load issues them (coalesced: every CTA reads the same lines), and
// gu_select_finish stores the keys, hands thread t the blocks [t * per,
// t * per + per) through shared memory (so one scan of the per-thread counts
// gives the block-id order), and selects with one barrier per radix pass and
// one per scan (block_select_reg, block_exclusive_scan_1b).
constexpr int kSelKeysPerThread = 8;
struct GuSelectSmem {
  RegSelectSmem sel;
  uint32_t keys[kSelKeysPerThread * 32 * 32];  // blockDim <= 1024
};
__device__ __forceinline__ void gu_select_load(const GateUpParams& p, float (&v)[kSelKeysPerThread]) {
#pragma unroll
  for (int j = 0; j < kSelKeysPerThread; ++j) {
    const int i = (int)threadIdx.x + j * (int)blockDim.x;
    v[j] = i < p.NB ? ldcg_f32(p.scores + i) : 0.f;
  }
}
__device__ __forceinline__ int gu_select_finish(const GateUpParams& p, const float (&v)[kSelKeysPerThread],
                                                GuSelectSmem& G, int* srows) {
  constexpr int KPT = kSelKeysPerThread;
  RegSelectSmem& S = G.sel;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = (int)(blockDim.x >> 5), NB = p.NB;
  uint32_t kor = 0u, kand = 0xffffffffu;
#pragma unroll
  for (int j = 0; j < KPT; ++j) {
    const int i = tid + j * (int)blockDim.x;
    if (i < NB) {
      const uint32_t key = orderable(v[j]);
      G.keys[i] = key;
      kor |= key;
      kand &= key;
    }
  }
  kor = __reduce_or_sync(0xffffffffu, kor);
  kand = __reduce_and_sync(0xffffffffu, kand);
  if (lane == 0) {
    S.s_or[warp] = kor;
    S.s_and[warp] = kand;
  }
  for (int i = tid; i < 512; i += (int)blockDim.x) (&S.hists[0][0])[i] = 0;
  __syncthreads();
  const uint32_t o = __reduce_or_sync(0xffffffffu, lane < nw ? S.s_or[lane] : 0u);
  const uint32_t a = __reduce_and_sync(0xffffffffu, lane < nw ? S.s_and[lane] : 0xffffffffu);
  const int per = (NB + (int)blockDim.x - 1) / (int)blockDim.x;  // <= KPT (the caller checks)
  const int lo = min(NB, tid * per), cnt = min(NB, lo + per) - lo;
  uint32_t key[KPT];
#pragma unroll
  for (int u = 0; u < KPT; ++u) key[u] = u < cnt ? G.keys[lo + u] : 0u;
  const RegSelection r = block_select_reg<KPT>(key, cnt, NB, p.top_k, o, a, S);
  int tot, eq_before = 0;
  if (r.split) {  // a tie at the threshold is split: rank the equal keys by block id
    int n_eq = 0;
#pragma unroll
    for (int u = 0; u < KPT; ++u) n_eq += u < cnt && key[u] == r.thr;
    eq_before = block_exclusive_scan_1b(n_eq, &tot, S.wtot[0]);
  }
  unsigned selmask = 0u;
  int m = 0;
#pragma unroll
  for (int u = 0, e = eq_before; u < KPT; ++u) {
    if (u < cnt) {
      const bool sel = key[u] > r.thr || (key[u] == r.thr && (!r.split || e++ < r.take_eq));
      if (sel && gu_map_block(p, lo + u) >= 0) {
        selmask |= 1u << u;
        ++m;
      }
    }
  }
  int pos = block_exclusive_scan_1b(m, &tot, S.wtot[1]);
#pragma unroll
  for (int u = 0; u < KPT; ++u) {
    if ((selmask >> u) & 1u) {
      const int row = gu_map_block(p, lo + u);
      srows[pos] = row;
      if (blockIdx.x == 0) {
        p.rows_out[pos] = row;
        p.row_block_out[pos] = lo + u;
      }
      ++pos;
    }
  }
  if (blockIdx.x == 0 && tid == 0) *p.count_out = tot;
  return tot;
}
static_assert(kGu1XloStageOff >= (int)sizeof(GuSelectSmem), "x16lo staging overlaps the selection scratch");
static_assert(kGu1Warps * kGuStages * kGuStageBytes >= (int)sizeof(GuSelectSmem) &&
                  kGuWarps * kGuStages * kGuStageBytes >= (int)sizeof(GuSelectSmem),
              "the register selection's scratch must fit in the gate/up ring");
static_assert(kGuWarps * kGuStages * kGuStageBytes >= kMaxNumBlocks * 4 + (int)sizeof(RadixSelectSmem),
              "the fused selection's keys must fit in the gate/up ring");
static_assert(kGu1Warps * kGuStages * kGuStageBytes >= kMaxNumBlocks * 4 + (int)sizeof(RadixSelectSmem),
              "the fused selection's keys must fit in the gate/up ring");

template <bool kOne>
__global__ void __launch_bounds__(GuCfg<kOne>::kWarps * 32, 1) gateup_tma_kernel(GateUpParams p) {
  using C = GuCfg<kOne>;
  char* smem = reinterpret_cast<char*>(g_lut_smem);
  const uint32_t bar0 = smem_u32(smem + C::kBarOff);
  const uint32_t xbar = bar0 + 8u * (uint32_t)(C::kWarps * kGuStages);
  if (threadIdx.x <= C::kWarps * kGuStages) mbar_init(bar0 + 8u * threadIdx.x, 1);
  mbar_init_fence();
  pdl_trigger();
  if (kOne) {
    // the caller declared the codebooks equal: check it (a mismatch is an
    // argument error, not a silently wrong up projection)
    const int diff = threadIdx.x < 16 && __ldg(p.gate_code + threadIdx.x) != __ldg(p.up_code + threadIdx.x);
    if (__syncthreads_or(diff)) {
      if (threadIdx.x == 0) record_error(p.err, NSM_ERR_INVALID_ARG);
      return;
    }
  }
  build_lut_alpha(p.gate_code, kOne ? p.gate_code : p.up_code, !kOne);
  pdl_wait();  // rows, count, x16 come from the router kernels
  __half* xs16 = reinterpret_cast<__half*>(smem + kGuX16Off);
  float* xss = reinterpret_cast<float*>(smem + C::kXsOff);
  int* srows = reinterpret_cast<int*>(smem + C::kRowsOff);
  const uint64_t xpol = l2_evict_last_policy();
  // the block selection's score loads leave before the x copies (they gate
  // the selection; every CTA reads the same lines)
  const bool reg_select = p.select && p.NB <= kSelKeysPerThread * (int)blockDim.x;
  float sv[kSelKeysPerThread];
  if (reg_select) gu_select_load(p, sv);
  // x16, x16lo and the x scales arrive by bulk copy while the block selection
  // runs (no thread waits on a global load before the selection); with a
  // shared codebook x16lo lands in the ring past the selection's scratch and
  // moves to the free table halves after it
  const bool xs_bulk = (p.H & 255) == 0;  // the scales' bytes (H / 16) a multiple of 16
  char* xlo_dst = kOne ? smem + C::kRingOff + kGu1XloStageOff : smem + kGuX16LoOff;
  if (threadIdx.x == 0) {
    fence_proxy_async_global();
    mbar_arrive_expect_tx(xbar, (uint32_t)p.H * 4u + (xs_bulk ? (uint32_t)p.H / 16u : 0u));
    bulk_g2s(smem_u32(xs16), p.x16, (uint32_t)p.H * 2u, xbar, xpol);
    bulk_g2s(smem_u32(xlo_dst), p.x16lo, (uint32_t)p.H * 2u, xbar, xpol);
    if (xs_bulk) bulk_g2s(smem_u32(xss), p.xscale, (uint32_t)p.H / 16u, xbar, xpol);
  }
  if (!xs_bulk)
    for (int i = threadIdx.x; i < p.H / 64; i += blockDim.x) xss[i] = __ldcg(p.xscale + i);
  const bool stage_rows = p.max_rows <= kStageRowsMax;
  int count;
  if (p.select) {
    // keys and selection scratch in the ring, which no copy has touched yet
    if (reg_select) {
      count = gu_select_finish(p, sv, *reinterpret_cast<GuSelectSmem*>(smem + C::kRingOff), srows);
    } else {
      uint32_t* keys = reinterpret_cast<uint32_t*>(smem + C::kRingOff);
      RadixSelectSmem* sel =
          reinterpret_cast<RadixSelectSmem*>(smem + C::kRingOff + (((size_t)p.NB * 4 + 127) & ~(size_t)127));
      count = gu_select_blocks(p, keys, *sel, srows);
    }
  } else {
    // the pool rows go out with the count (up to the capacity; rows past the
    // count are never read)
    count = *p.count_ptr;
    if (stage_rows)
      for (int i = threadIdx.x; i < p.max_rows; i += blockDim.x) srows[i] = __ldcg(p.rows + i);
  }
  // shared codebook: every thread waits for the copies and moves its chunks
  // of x16lo into the table holes (the ring is free until the next barrier)
  bool x_late = false;
  if ((kOne || threadIdx.x == 0) && !mbar_wait(xbar, 0, p.wait_spins)) {
    record_error(p.err, NSM_ERR_TIMEOUT);
    mbar_wait(xbar, 0);  // the copies land before the CTA leaves
    x_late = true;
  }
  if (kOne && !x_late)
    for (int i = threadIdx.x; i < p.H / 8; i += blockDim.x)
      *reinterpret_cast<uint4*>(smem + gu1_xlo_off(i >> 3, i & 7)) = reinterpret_cast<const uint4*>(xlo_dst)[i];
  if (__syncthreads_or(x_late)) return;
  const int* rows = stage_rows ? srows : p.rows;
  const uint32_t lb = (threadIdx.x & 31) * 4u;
  const uint32_t ring = smem_u32(smem + C::kRingOff);
  const uint32_t xlo_s = kOne ? smem_u32(smem) : smem_u32(smem + kGuX16LoOff);
  if (lut_base_addr() == 0x400u)
    gateup_tma_body<0x400, kOne>(p, lb, smem_u32(xs16), xlo_s, smem_u32(xss), rows, count, ring, bar0);
  else
    gateup_tma_body<-1, kOne>(p, lb, smem_u32(xs16), xlo_s, smem_u32(xss), rows, count, ring, bar0);
}

// Down, bulk-copy variant: a pair is (64-row group rp, slot s) = two adjacent
// 32-row tiles of one block (1 KB packed + 256 B absmax, contiguous in the
// tiled layout); pairs are rp-major.  A stage holds kDnPairsPerStage pairs.
template <int kBase>
__device__ __forceinline__ void down_tma_body(const DownParams& p, uint32_t lb, uint32_t shi_s, uint32_t slo_s,
                                              uint32_t sscale_s, const int* rows, int count, uint32_t ring,
                                              uint32_t bar0) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  // B operand column 0 (lanes g == 0) is act16, column 1 (lanes g == 1) act16lo
  const uint32_t sact_s = g == 1 ? slo_s : shi_s;
  const float ia = lut_inv_alpha(0);
  const int warp = threadIdx.x >> 5;
  const int warp_global = blockIdx.x * kTmaWarps + warp;
  const int RP = p.H >> 6;
  const int total = RP * count;
  const int nw = stream_warps(RP, count, kMaxSlotGroups, p.total_warps);
  if (warp_global >= nw) return;
  const int q0 = stream_begin(total, nw, warp_global), q1 = stream_begin(total, nw, warp_global + 1);
  const uint32_t wring = ring + (uint32_t)(warp * kDnStages * kDnStageBytes);
  const uint32_t wbar = bar0 + (uint32_t)(warp * kDnStages * 8);
  const uint64_t pol = l2_evict_first_policy();
  int lrp = q0 / count, ls = q0 - lrp * count;  // load cursor
  int lq = q0;
  int issued = 0;
  auto issue_next = [&](int stage) {  // up to kDnPairsPerStage pairs into `stage`
    ++issued;
    const int n = min(kDnPairsPerStage, q1 - lq);
    if (lane == 0) {
      fence_proxy_async_smem();  // the warp's reads of this stage come first
      const uint32_t dst = wring + (uint32_t)(stage * kDnStageBytes);
      const uint32_t bar = wbar + 8u * (uint32_t)stage;
      mbar_arrive_expect_tx(bar, (uint32_t)n * 1280u);
      int rp = lrp, sl = ls;
      for (int i = 0; i < n; ++i) {
        const int prow = rows[sl];
        bulk_g2s(dst + i * 1024, p.down + (int64_t)prow * p.dbs + (int64_t)rp * 1024, 1024u, bar, pol);
        bulk_g2s(dst + kDnPairsPerStage * 1024 + i * 256, p.down_am + (int64_t)prow * p.dabs + rp * 64, 256u, bar,
                 pol);
        if (++sl == count) { sl = 0; ++rp; }
      }
    }
    lq += n;
    ls += n;
    while (ls >= count) { ls -= count; ++lrp; }
  };
#pragma unroll
  for (int i = 0; i < kDnStages; ++i)
    if (q0 + i * kDnPairsPerStage < q1) issue_next(i);

  int rp = q0 / count, s = q0 - rp * count;
  int seg = warp_global - stream_owner(total, nw, rp * count);
  float acc[2][4] = {};  // tile r of the group: rows g, g+8, 16+g, 24+g
  uint32_t phase = 0;
  int q = q0;
  bool ok = true;
  while (q < q1 && ok) {
#pragma unroll
    for (int st = 0; st < kDnStages; ++st) {
      if (q < q1 && ok) {
        if (!mbar_wait(wbar + 8u * st, phase, p.wait_spins)) {
          ok = false;
        } else {
          const uint32_t sb = wring + (uint32_t)(st * kDnStageBytes);
#pragma unroll
          for (int i = 0; i < kDnPairsPerStage; ++i) {
            if (q < q1) {
              const uint4 w0 = lds_u4(sb + i * 1024 + lane * 16);
              const uint4 w1 = lds_u4(sb + i * 1024 + 512 + lane * 16);
              const float4 a0 = lds_f4(sb + kDnPairsPerStage * 1024 + i * 256 + g * 16);
              const float4 a1 = lds_f4(sb + kDnPairsPerStage * 1024 + i * 256 + 128 + g * 16);
              const uint4 bf = lds_u4(sact_s + (uint32_t)(s * 64 + t * 16));
              float as;
              asm volatile("ld.shared.f32 %0, [%1];" : "=f"(as) : "r"(sscale_s + (uint32_t)(s * 4)));
              as *= ia;
              float d[4];
              down_mma<kBase>(lb, w0.x, w0.y, bf, d);
              acc[0][0] = fmaf(d[0] + d[1], a0.x * as, acc[0][0]);
              acc[0][1] = fmaf(d[2] + d[3], a0.y * as, acc[0][1]);
              down_mma<kBase>(lb, w0.z, w0.w, bf, d);
              acc[0][2] = fmaf(d[0] + d[1], a0.z * as, acc[0][2]);
              acc[0][3] = fmaf(d[2] + d[3], a0.w * as, acc[0][3]);
              down_mma<kBase>(lb, w1.x, w1.y, bf, d);
              acc[1][0] = fmaf(d[0] + d[1], a1.x * as, acc[1][0]);
              acc[1][1] = fmaf(d[2] + d[3], a1.y * as, acc[1][1]);
              down_mma<kBase>(lb, w1.z, w1.w, bf, d);
              acc[1][2] = fmaf(d[0] + d[1], a1.z * as, acc[1][2]);
              acc[1][3] = fmaf(d[2] + d[3], a1.w * as, acc[1][3]);
              ++q;
              if (++s == count || q == q1) {
                if (t == 0) {
                  float* yp = p.ypart + (int64_t)seg * p.H + rp * 64;
#pragma unroll
                  for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int c = 0; c < 4; ++c) yp[r * 32 + (c >> 1) * 16 + g + (c & 1) * 8] = acc[r][c];
                }
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                  for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
                seg = 0;  // this warp holds the first pair of the next group
                if (s == count) { s = 0; ++rp; }
              }
            }
          }
          __syncwarp();
          if (lq < q1) issue_next(st);
        }
      }
    }
    phase ^= 1u;
  }
  if (!ok) {
    record_error(p.err, NSM_ERR_TIMEOUT);
    drain_ring<kDnStages>(wbar, (q - q0) / kDnPairsPerStage, issued);
  }
}

__global__ void __launch_bounds__(kTmaThreads, 1) down_tma_kernel(DownParams p) {
  char* smem = reinterpret_cast<char*>(g_lut_smem);
  const uint32_t bar0 = smem_u32(smem + kDnBarOff);
  const uint32_t abar = bar0 + 8u * (uint32_t)(kTmaWarps * kDnStages);
  if (threadIdx.x <= kTmaWarps * kDnStages) mbar_init(bar0 + 8u * threadIdx.x, 1);
  mbar_init_fence();
  pdl_trigger();
  build_lut_alpha(p.down_code, p.down_code, false);  // the down loops read table 0 only
  pdl_wait();  // act16 / act_scale come from the gate/up kernels
  record_down_meta(p);
  __half* sact = reinterpret_cast<__half*>(smem + kDnActOff);
  __half* sactlo = reinterpret_cast<__half*>(smem + kDnActLoOff);
  float* sscale = reinterpret_cast<float*>(smem + kDnScaleOff);
  int* srows = reinterpret_cast<int*>(smem + kDnRowsOff);
  // staged up to the capacity, with the count (entries past it are never
  // read), all on one barrier: act16 / act16lo, and the scales and rows when
  // their bytes are whole 16-byte runs (else plain loads); no thread waits on
  // a global load before the staging is in flight
  const bool sr_bulk = (p.max_rows & 3) == 0 && (((uintptr_t)p.act_scale | (uintptr_t)p.rows) & 15) == 0;
  if (threadIdx.x == 0) {
    const uint64_t pol = l2_evict_last_policy();
    fence_proxy_async_global();
    mbar_arrive_expect_tx(abar, (uint32_t)p.max_rows * (sr_bulk ? 136u : 128u));
    bulk_g2s(smem_u32(sact), p.act16, (uint32_t)p.max_rows * 64u, abar, pol);
    bulk_g2s(smem_u32(sactlo), p.act16lo, (uint32_t)p.max_rows * 64u, abar, pol);
    if (sr_bulk) {
      bulk_g2s(smem_u32(sscale), p.act_scale, (uint32_t)p.max_rows * 4u, abar, pol);
      bulk_g2s(smem_u32(srows), p.rows, (uint32_t)p.max_rows * 4u, abar, pol);
    }
  }
  const int count = __ldcg(p.count_ptr);
  if (!sr_bulk)
    for (int i = threadIdx.x; i < p.max_rows; i += blockDim.x) {
      sscale[i] = __ldcg(p.act_scale + i);
      srows[i] = __ldcg(p.rows + i);
    }
  bool a_late = false;
  if (threadIdx.x == 0 && !mbar_wait(abar, 0, p.wait_spins)) {
    record_error(p.err, NSM_ERR_TIMEOUT);
    mbar_wait(abar, 0);  // the copies land before the CTA leaves
    a_late = true;
  }
  if (__syncthreads_or(a_late)) return;
  const uint32_t lb = (threadIdx.x & 31) * 4u;
  const uint32_t ring = smem_u32(smem + kDnRingOff);
  if (lut_base_addr() == 0x400u)
    down_tma_body<0x400>(p, lb, smem_u32(sact), smem_u32(sactlo), smem_u32(sscale), srows, count, ring, bar0);
  else
    down_tma_body<-1>(p, lb, smem_u32(sact), smem_u32(sactlo), smem_u32(sscale), srows, count, ring, bar0);
}

// ============================================================================
// host side
// ============================================================================
static int dtype_ok(int d) { return d == NSM_F32 || d == NSM_F16 || d == NSM_BF16; }

constexpr int kGateupSmem = kSmemHead + kStageRowsMax * 4;
constexpr int kGateupSmemStaged = kGateupSmem + kStageXMaxHidden * 2 + (kStageXMaxHidden / 64) * 4;
constexpr int kDownSmemStaged = kSmemHead + kStageActMaxSlots * (64 + 4 + 4 + 64);

struct KernelSetup {
  bool done = false;
  int gu[2][2] = {{0, 0}, {0, 0}};  // [tiled][staged] CTAs per SM
  int dn[2][2] = {{0, 0}, {0, 0}};
  int gu_tma = 0;  // CTAs per SM of the bulk-copy variants (1 when they fit)
  int gu_tma1 = 0;  // ... of the shared-codebook gate/up variant
  int dn_tma = 0;
};
static KernelSetup g_setup[64];

template <typename K>
static int setup_one(K kernel, int smem, int* ctas_per_sm, int threads = kMlpThreads) {
  NSM_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  NSM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, kernel, threads, smem));
  if (*ctas_per_sm <= 0) return fail(NSM_ERR_CUDA, "kernel occupancy is zero");
  return NSM_OK;
}

static int setup_kernels(const DeviceInfo& d, KernelSetup** out) {
  KernelSetup& s = g_setup[d.device];
  if (!s.done) {
    int st = setup_one(gateup_kernel<false, false>, kGateupSmem, &s.gu[0][0]);
    if (!st) st = setup_one(gateup_kernel<false, true>, kGateupSmemStaged, &s.gu[0][1]);
    if (!st) st = setup_one(gateup_kernel<true, false>, kGateupSmem, &s.gu[1][0]);
    if (!st) st = setup_one(gateup_kernel<true, true>, kGateupSmemStaged, &s.gu[1][1]);
    if (!st) st = setup_one(down_kernel<false, false>, kSmemHead, &s.dn[0][0]);
    if (!st) st = setup_one(down_kernel<false, true>, kDownSmemStaged, &s.dn[0][1]);
    if (!st) st = setup_one(down_kernel<true, false>, kSmemHead, &s.dn[1][0]);
    if (!st) st = setup_one(down_kernel<true, true>, kDownSmemStaged, &s.dn[1][1]);
    if (!st) st = setup_one(gateup_tma_kernel<false>, kGuTmaSmem, &s.gu_tma, kGuThreads);
    if (!st) st = setup_one(gateup_tma_kernel<true>, kGu1TmaSmem, &s.gu_tma1, kGu1Threads);
    if (!st) st = setup_one(down_tma_kernel, kDnTmaSmem, &s.dn_tma, kTmaThreads);
    if (!st) st = router_setup();
    if (st) return st;
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
  void* const* events;  // optional NSM_STAGE_EVENTS stage events (index 1..5 recorded here)
  bool defer_y;         // leave the output as down partials in the workspace
  // select: the gate/up kernel selects the blocks from ws.scores (no top-k kernel)
  bool select;
  int NB;
  const nsm_block_map* map;
};

static cudaError_t stage_event(void* const* ev, int i, cudaStream_t s) {
  return ev != nullptr ? cudaEventRecord(reinterpret_cast<cudaEvent_t>(ev[i]), s) : cudaSuccess;
}

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

// The bulk-copy gate/up kernel applies: tiled pools, the x vector staged in
// shared memory, 16-byte aligned pools and strides, whole two-tile units.
static bool gateup_tma_ok(const nsm_mlp_weights* w, int H, const KernelSetup* ks) {
  const int64_t gstride = w->gateup_block_stride ? w->gateup_block_stride : (int64_t)16 * H;
  const int64_t gastride = w->gateup_absmax_block_stride ? w->gateup_absmax_block_stride : (int64_t)H / 2;
  const bool aligned = ((uintptr_t)w->gate_packed | (uintptr_t)w->up_packed | (uintptr_t)w->gate_absmax |
                        (uintptr_t)w->up_absmax) % 16 == 0 &&
                       gstride % 16 == 0 && (gastride * 4) % 16 == 0;
  return (w->layout & NSM_LAYOUT_GATEUP_TILED) != 0 && H <= kStageXMaxHidden && aligned && ks->gu_tma > 0 &&
         (H / 64) % kGuUnitTiles == 0;
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
  gp.max_rows = m.k;
  gp.row_block = m.row_block;
  gp.x16 = ws.x16;
  gp.x16lo = ws.x16lo;
  gp.xscale = ws.xscale;
  gp.norm_scale = m.norm_scale;
  gp.act_mask = m.act_mask;
  gp.mask_dtype = m.mask_dtype;
  gp.gu_part = ws.gu_part;
  gp.err = ws.err;
  gp.act16 = ws.act16;
  gp.act16lo = ws.act16lo;
  gp.act_scale = ws.act_scale;
  gp.act_out = m.act_out;
  gp.wait_spins = copy_wait_spins();
  const bool gu_tiled = (w->layout & NSM_LAYOUT_GATEUP_TILED) != 0;
  const bool gu_stage = m.H <= kStageXMaxHidden;
  const bool gu_tma = gateup_tma_ok(w, m.H, ks);
  if (m.select) {
    NSM_REQUIRE(gu_tma, NSM_ERR_INVALID_ARG, "the fused block selection needs the bulk-copy gate/up kernel");
    gp.select = 1;
    gp.scores = ws.scores;
    gp.NB = m.NB;
    gp.top_k = m.k;
    gp.slot_of_block = m.map ? m.map->slot_of_block : nullptr;
    gp.block_begin = m.map ? m.map->block_begin : 0;
    gp.block_end = m.map ? m.map->block_end : m.NB;
    gp.pool_rows = w->pool_rows;
    gp.rows_out = ws.rows;
    gp.row_block_out = ws.row_block;
    gp.count_out = ws.count;
  }
  NSM_CHECK_CUDA(stage_event(m.events, 1, stream));
  cudaError_t e;
  gp.unit_tiles = 1;
  if (gu_tma) {
    const bool one = (w->layout & NSM_LAYOUT_SHARED_CODE) != 0 && ks->gu_tma1 > 0;
    gp.unit_tiles = kGuUnitTiles;
    gp.total_warps = dev.sm_count * (one ? kGu1Warps : kGuWarps);
    gp.fused_finalize = 1;
    gp.gu_ticket = ws.gu_ticket;
    if (one) e = launch_pdl(gateup_tma_kernel<true>, dev.sm_count, kGu1Threads, kGu1TmaSmem, stream, gp);
    else e = launch_pdl(gateup_tma_kernel<false>, dev.sm_count, kGuThreads, kGuTmaSmem, stream, gp);
  } else {
  const int gu_ctas = dev.sm_count * ks->gu[gu_tiled][gu_stage];
  gp.total_warps = gu_ctas * (kMlpThreads / 32);
  const int gu_smem = gu_stage ? kGateupSmemStaged : kGateupSmem;
  if (gu_tiled) {
    if (gu_stage) e = launch_pdl(gateup_kernel<true, true>, gu_ctas, kMlpThreads, gu_smem, stream, gp);
    else e = launch_pdl(gateup_kernel<true, false>, gu_ctas, kMlpThreads, gu_smem, stream, gp);
  } else {
    if (gu_stage) e = launch_pdl(gateup_kernel<false, true>, gu_ctas, kMlpThreads, gu_smem, stream, gp);
    else e = launch_pdl(gateup_kernel<false, false>, gu_ctas, kMlpThreads, gu_smem, stream, gp);
  }
  }
  NSM_CHECK_CUDA(e);
  NSM_CHECK_CUDA(stage_event(m.events, 2, stream));
  if (!gp.fused_finalize) NSM_CHECK_CUDA(launch_pdl(gateup_finalize_kernel, m.k, 256, 0, stream, gp));
  NSM_CHECK_CUDA(stage_event(m.events, 3, stream));

  DownParams dp{};
  dp.down = w->down_packed;
  dp.down_am = w->down_absmax;
  const bool dn_tiled_layout = (w->layout & NSM_LAYOUT_DOWN_TILED) != 0;
  dp.dbs = w->down_block_stride ? w->down_block_stride : (int64_t)16 * m.H;
  dp.drs = (w->down_row_stride && !dn_tiled_layout) ? w->down_row_stride : 16;
  dp.dabs = w->down_absmax_block_stride ? w->down_absmax_block_stride : (int64_t)m.H;
  dp.dars = (w->down_absmax_row_stride && !dn_tiled_layout) ? w->down_absmax_row_stride : 1;
  dp.pair = (w->layout & NSM_LAYOUT_DOWN_TILED) ? 0 : w->down_absmax_pair;
  dp.down_code = w->down_code;
  dp.down_bias = w->down_bias;
  dp.bias_dtype = w->bias_dtype;
  dp.H = m.H;
  dp.rows = m.rows;
  dp.count_ptr = m.count;
  dp.max_rows = m.k;
  dp.act16 = ws.act16;
  dp.act16lo = ws.act16lo;
  dp.act_scale = ws.act_scale;
  dp.ypart = ws.ypart;
  dp.err = ws.err;
  dp.y = m.y;
  dp.y_dtype = m.y_dtype;
  dp.wait_spins = copy_wait_spins();
  const bool dn_tiled = (w->layout & NSM_LAYOUT_DOWN_TILED) != 0;
  const bool dn_stage = m.k <= kStageActMaxSlots;
  const bool dn_aligned = ((uintptr_t)dp.down | (uintptr_t)dp.down_am) % 16 == 0 && dp.dbs % 16 == 0 &&
                          (dp.dabs * 4) % 16 == 0;
  const bool dn_tma = dn_tiled && dn_stage && dn_aligned && ks->dn_tma > 0;
  dp.group_log2 = dn_tma ? 6 : 5;
  dp.meta = ws.down_meta;
  if (dn_tma) {
    dp.total_warps = dev.sm_count * kTmaWarps;
    e = launch_pdl(down_tma_kernel, dev.sm_count, kTmaThreads, kDnTmaSmem, stream, dp);
  } else {
  const int dn_ctas = dev.sm_count * ks->dn[dn_tiled][dn_stage];
  dp.total_warps = dn_ctas * (kMlpThreads / 32);
  const int dn_smem = dn_stage ? kDownSmemStaged : kSmemHead;
  if (dn_tiled) {
    if (dn_stage) e = launch_pdl(down_kernel<true, true>, dn_ctas, kMlpThreads, dn_smem, stream, dp);
    else e = launch_pdl(down_kernel<true, false>, dn_ctas, kMlpThreads, dn_smem, stream, dp);
  } else {
    if (dn_stage) e = launch_pdl(down_kernel<false, true>, dn_ctas, kMlpThreads, dn_smem, stream, dp);
    else e = launch_pdl(down_kernel<false, false>, dn_ctas, kMlpThreads, dn_smem, stream, dp);
  }
  }
  NSM_CHECK_CUDA(e);
  NSM_CHECK_CUDA(stage_event(m.events, 4, stream));
  if (!m.defer_y) NSM_CHECK_CUDA(launch_pdl(down_finalize_kernel, (4 * m.H + 255) / 256, 256, 0, stream, dp));
  NSM_CHECK_CUDA(stage_event(m.events, 5, stream));
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

static RouterAParams router_a_params(const void* x, int x_dtype, const nsm_layer_io* io,
                                     const nsm_router_weights* rw, int H, const DecodeWs& ws) {
  RouterAParams a{};
  a.x = x;
  a.x_dtype = x_dtype;
  if (io && io->residual) {
    a.residual = io->residual;
    a.pending = (io->flags & NSM_IO_PENDING_Y) != 0;
    if (a.pending && io->exchange) a.ex = *exchange_dev(io->exchange);
    a.y_prev = a.pending ? nullptr : io->y_prev;
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
  a.ws = ws;
  return a;
}

static int router_a_prepare(const void* x, int x_dtype, const nsm_layer_io* io, const nsm_router_weights* rw,
                            int H, const DecodeWs& ws, cudaStream_t stream) {
  return router_a_launch(router_a_params(x, x_dtype, io, rw, H, ws), stream);
}

// Router kernel + scores/top-k kernels; the scores kernel reduces the router
// kernel's partial latents (and advances the exchange epoch).
static int router_launch_pair(const RouterAParams& a_in, RouterBParams b, cudaStream_t stream, bool topk = true) {
  RouterAParams a = a_in;
  a.reduce_in_scores = 1;
  int cpc;
  b.reduce_latent = 1;
  b.nparts = router_a_ctas(a.H, &cpc);
  b.use_norm = a.use_norm;
  b.eps = a.eps;
  b.H = a.H;
  b.enc_b = a.enc_b;
  b.basis_top_k = a.basis_top_k;
  b.epoch_counter = (a.pending && a.ex.world > 1) ? a.ex.counter : nullptr;
  int st = router_a_launch(a, stream);
  if (st) return st;
  return router_b_launch(b, stream, topk);
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

static RouterBParams router_b_params(const nsm_router_weights* rw, int k, int32_t* idx_out, float* score_out,
                                     float* latent_out, const nsm_block_map* map, int pool_rows,
                                     const DecodeWs& ws) {
  RouterBParams b{};
  b.score_w = rw->score_w;
  b.score_b = rw->score_b;
  b.wdtype = rw->weight_dtype;
  b.dbn = rw->down_block_norm;
  b.legacy = rw->legacy_abs_latent;
  b.rank = rw->rank;
  b.NB = rw->num_blocks;
  b.top_k = k;
  b.idx_out = idx_out;
  b.score_out = score_out;
  b.latent_out = latent_out;
  b.slot_of_block = map ? map->slot_of_block : nullptr;
  b.block_begin = map ? map->block_begin : 0;
  b.block_end = map ? map->block_end : b.NB;
  b.pool_rows = pool_rows;
  b.ws = ws;
  return b;
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
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
  NSM_REQUIRE(idx_out != nullptr, NSM_ERR_INVALID_ARG, "idx_out is NULL");
  const int k = std::max(1, std::min(rw->top_k, rw->num_blocks));
  NSM_REQUIRE(k <= kMaxTopK, NSM_ERR_UNSUPPORTED, "top_k too large");
  const int I = rw->num_blocks * 32;
  const size_t need = decode_ws_layout(nullptr, hidden, I, k, rw->rank).bytes;
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "nsm_route: workspace missing, not 256-byte aligned or too small");
  DecodeWs w = decode_ws_layout(ws, hidden, I, k, rw->rank);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  return router_launch_pair(router_a_params(x, x_dtype, nullptr, rw, hidden, w),
                            router_b_params(rw, k, idx_out, score_out, latent_out, nullptr, rw->num_blocks, w), s);
}

int nsm_route_rows(const void* x, int32_t x_dtype, int32_t rows, int32_t hidden, const nsm_router_weights* rw,
                   int32_t* idx_out, float* score_out, float* latent_out, void* ws, size_t ws_bytes,
                   nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  st = validate_router(rw, hidden);
  if (st) return st;
  NSM_REQUIRE(x != nullptr && dtype_ok(x_dtype), NSM_ERR_INVALID_ARG, "x is NULL or has a bad dtype");
  NSM_REQUIRE(rows > 0 && rows <= 65535, NSM_ERR_UNSUPPORTED, "rows must be in [1, 65535]");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
  NSM_REQUIRE(idx_out != nullptr, NSM_ERR_INVALID_ARG, "idx_out is NULL");
  const int k = std::max(1, std::min(rw->top_k, rw->num_blocks));
  NSM_REQUIRE(k <= kMaxTopK, NSM_ERR_UNSUPPORTED, "top_k too large");
  const int I = rw->num_blocks * 32;
  const size_t need = decode_ws_layout(nullptr, hidden, I, k, rw->rank, rows).bytes;
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "nsm_route_rows: workspace missing, not 256-byte aligned or too small");
  DecodeWs w = decode_ws_layout(ws, hidden, I, k, rw->rank, rows);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  return router_rows_launch(router_a_params(x, x_dtype, nullptr, rw, hidden, w),
                            router_b_params(rw, k, idx_out, score_out, latent_out, nullptr, rw->num_blocks, w), rows,
                            reinterpret_cast<cudaStream_t>(stream));
}

int nsm_sparse_mlp_decode(const void* x, int32_t x_dtype, int32_t hidden, int32_t intermediate,
                          const nsm_layer_io* io, const nsm_router_weights* rw, const int32_t* idx_in, int32_t k_in,
                          const nsm_block_map* map, const nsm_mlp_weights* w, void* y, int32_t y_dtype,
                          int32_t* idx_out, float* score_out, void* ws, size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
  NSM_REQUIRE(intermediate > 0 && intermediate % 64 == 0, NSM_ERR_UNSUPPORTED,
              "intermediate must be a positive multiple of 64");
  const bool resid = io != nullptr && io->residual != nullptr;
  NSM_REQUIRE(resid || (x != nullptr && dtype_ok(x_dtype)), NSM_ERR_INVALID_ARG, "x is NULL or has a bad dtype");
  if (resid && io->y_prev) NSM_REQUIRE(dtype_ok(io->y_prev_dtype), NSM_ERR_INVALID_ARG, "bad y_prev dtype");
  if (resid && io->norm_weight)
    NSM_REQUIRE(dtype_ok(io->norm_weight_dtype), NSM_ERR_INVALID_ARG, "bad norm weight dtype");
  const bool defer = io != nullptr && (io->flags & NSM_IO_DEFER_Y) != 0;
  NSM_REQUIRE(defer || (y != nullptr && dtype_ok(y_dtype)), NSM_ERR_INVALID_ARG, "y is NULL or has a bad dtype");
  if (io && (io->flags & NSM_IO_PENDING_Y)) NSM_REQUIRE(resid, NSM_ERR_INVALID_ARG, "NSM_IO_PENDING_Y needs io->residual");
  if (io && io->exchange) NSM_REQUIRE(exchange_dev(io->exchange)->hidden == hidden && exchange_dev(io->exchange)->data[0],
                                      NSM_ERR_INVALID_ARG, "exchange not connected or built for another hidden size");
  st = validate_weights(w, hidden);
  if (st) return st;
  if (defer) NSM_REQUIRE(w->down_bias == nullptr, NSM_ERR_UNSUPPORTED, "NSM_IO_DEFER_Y needs a down projection without bias");
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
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "nsm_sparse_mlp_decode: workspace missing, not 256-byte aligned or too small");
  DecodeWs wsl = decode_ws_layout(ws, hidden, intermediate, k, rank);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;

  void* const* events = io != nullptr ? io->stage_events : nullptr;
  NSM_CHECK_CUDA(stage_event(events, 0, s));
  // the gate/up kernel selects the blocks itself (no top-k kernel) when nobody
  // asks for the ordered indices and the bulk-copy kernel applies
  const bool fuse_select = idx_in == nullptr && idx_out == nullptr && score_out == nullptr && k <= kStageRowsMax &&
                           NB <= kMaxNumBlocks && gateup_tma_ok(w, hidden, ks);
  if (idx_in == nullptr) {
    st = router_launch_pair(router_a_params(x, x_dtype, io, rw, hidden, wsl),
                            router_b_params(rw, k, idx_out, score_out, nullptr, map, w->pool_rows, wsl), s,
                            !fuse_select);
    if (st) return st;
  } else {
    st = router_a_prepare(x, x_dtype, io, nullptr, hidden, wsl, s);
    if (st) return st;
    RouterBParams b{};
    b.NB = NB;
    b.slot_of_block = map ? map->slot_of_block : nullptr;
    b.block_begin = map ? map->block_begin : 0;
    b.block_end = map ? map->block_end : NB;
    b.pool_rows = w->pool_rows;
    b.ws = wsl;
    st = select_given_launch(b, idx_in, k, s);
    if (st) return st;
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
  m.events = events;
  m.defer_y = defer;
  m.select = fuse_select;
  m.NB = NB;
  m.map = map;
  return launch_mlp(m, wsl, s);
}

int nsm_residual_flush(int32_t hidden, const nsm_layer_io* io, void* ws, size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
  NSM_REQUIRE(io != nullptr && io->residual != nullptr && (io->flags & NSM_IO_PENDING_Y), NSM_ERR_INVALID_ARG,
              "nsm_residual_flush needs io->residual and NSM_IO_PENDING_Y");
  if (io->exchange) NSM_REQUIRE(exchange_dev(io->exchange)->hidden == hidden && exchange_dev(io->exchange)->data[0],
                                NSM_ERR_INVALID_ARG, "exchange not connected or built for another hidden size");
  const size_t need = decode_ws_layout(nullptr, hidden, 64, 1, 1).bytes;
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "nsm_residual_flush: workspace missing, not 256-byte aligned or too small");
  DecodeWs wsl = decode_ws_layout(ws, hidden, 64, 1, 1);
  return router_a_prepare(nullptr, 0, io, nullptr, hidden, wsl, reinterpret_cast<cudaStream_t>(stream));
}

int nsm_decode_gathered(const void* x, int32_t x_dtype, int32_t hidden, int32_t num_blocks_gathered,
                        const nsm_mlp_weights* w, void* y, int32_t y_dtype, float* act_out, void* ws,
                        size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
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
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "nsm_decode_gathered: workspace missing, not 256-byte aligned or too small");
  DecodeWs wsl = decode_ws_layout(ws, hidden, I, k, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  st = router_a_prepare(x, x_dtype, nullptr, nullptr, hidden, wsl, s);
  if (st) return st;
  NSM_CHECK_CUDA(launch_pdl(identity_rows_kernel, (k + 255) / 256, 256, 0, s, wsl.rows, wsl.count, wsl.sel_idx, k));
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
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED,
              "hidden must be a positive multiple of 64, at most 65536");
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
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= need, NSM_ERR_WORKSPACE, "workspace missing, not 256-byte aligned or too small");
  DecodeWs wsl = decode_ws_layout(ws, hidden, I, k, 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  KernelSetup* ks;
  st = setup_kernels(dev, &ks);
  if (st) return st;
  NSM_CHECK_CUDA(launch_pdl(identity_rows_kernel, (k + 255) / 256, 256, 0, s, wsl.rows, wsl.count, wsl.sel_idx, k));
  const int xes = x_dtype == NSM_F32 ? 4 : 2;
  const int yes = y_dtype == NSM_F32 ? 4 : 2;
  const int mes = mask_dtype == NSM_F32 ? 4 : 2;
  for (int r = 0; r < rows; ++r) {
    st = router_a_prepare(reinterpret_cast<const char*>(x) + (size_t)r * hidden * xes, x_dtype, nullptr, nullptr,
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
