// nsm_lmhead.cu -- NF4 LM head: a dense NF4 GEMV over a bitsandbytes
// row-major weight W [V, H] for 1..8 tokens (the reference's GPU NF4 LM head,
// llama3_neuroplastic/experiments/runtime/lm_head.py:267-468).
//
//   logits[t][v] = sum_h code[nib(v*H + h)] * absmax[(v*H + h) / qbs] * x[t][h]  (+ bias[v])
//
// This is the math of the reference's dense LM head (F.linear on the
// dequantised weight, lm_head.py:472-480).  The reference's NF4 path hands the
// same row-major bytes to triton_sparse_input_linear_4bit, whose kernels index
// the weight as weight.t() (triton_sparse_mlp.py:495-496), so on a GPU its NF4
// logits are not its dense logits; the dense head's math is the one kept here.
//
// Three launches:
//  1. lmhead_prep_kernel: per token a power-of-two scale s with max|x|/s in
//     [2^14, 2^15), x/s as fp16 into the workspace (exact for bf16 / fp16
//     inputs; the fp16 products below cannot overflow) and s;
//  2. lmhead_gemv_kernel: persistent, one CTA of 16 warps per SM.  A work
//     unit is 16 rows (one m16 tile) x a run of 64-column chunks (split-K).
//     Each warp streams its unit through its own 3-stage cp.async ring; a
//     stage is 4 chunks: 16 rows x one 128-byte line (so every copy
//     instruction moves whole lines: the copy cost scales with the lines
//     touched) plus the rows' 4 absmax, with the 16-byte granules of a row
//     XOR-swizzled by the row so the fragment reads are conflict-free.  It
//     dequantises with the per-lane byte->half2 table (one prmt and one
//     conflict-free shared load per byte) and accumulates with mma.sync
//     m16n8k16 (f16 x f16 -> f32): A = 16 rows x 16 permuted columns of W,
//     B = the same 16 columns of x for 8 token slots.  A chunk's four MMAs
//     cover exactly one absmax group per row, so the group's scale is applied
//     in fp32 after them.  fp32 partials [split][token][V] (deterministic);
//  3. lmhead_finalize_kernel: sum of the splits, times s, + bias, output dtype.
//
// Streams HBM-bound: 0.5625 B of weight + absmax per (row, column) at qbs 64.
// No waits other than cp.async.wait_group on the warp's own copies.
#include <algorithm>
#include <mutex>

#include "nsm_common.cuh"
#include "nsm_internal.h"

namespace nsm {
namespace {

constexpr int kLhWarps = 16;
constexpr int kLhThreads = 32 * kLhWarps;
constexpr int kLhRows = 16;                           // one m16 row tile per unit
constexpr int kLhSc = 4;                              // 64-column chunks per ring stage
constexpr int kLhRowBytes = 32 * kLhSc;               // one row's bytes per stage (a 128 B line)
constexpr int kLhStages = 3;
constexpr int kLhStageBytes = kLhRows * kLhRowBytes + kLhRows * kLhSc * 4;  // 16 x 128 B + absmax
constexpr int kLhRingBytes = kLhWarps * kLhStages * kLhStageBytes;
constexpr int kLhMaxTokens = 8;
constexpr int kLhUnitsPerWarp = 8;                    // split-K target for load balance

struct LmHeadParams {
  const __half* xh;       // [T][H] fp16, x / s
  const uint8_t* packed;  // [V*H/2]
  const float* absmax;    // [V*H/qbs]
  const float* code;      // [16]
  float* part;            // [splits][T][V]
  int xs_bytes;           // staged x, 16-byte multiple
  int T, V, H, qbs;
  int splits, cps, nchunks;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint2 lds_u2(uint32_t addr) {
  uint2 r;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(addr));
  return r;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float r;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"(addr));
  return r;
}

__global__ void __launch_bounds__(1024) lmhead_prep_kernel(const void* x, int dt, int H, __half* xh, float* scale) {
  __shared__ float wmax[32];
  const int t = blockIdx.x;
  float m = 0.f;
  for (int h = threadIdx.x; h < H; h += blockDim.x) m = fmaxf(m, fabsf(load_as_f32(x, dt, (int64_t)t * H + h)));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? wmax[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) wmax[0] = v;
  }
  __syncthreads();
  const float s = pow2_scale_for(wmax[0]);
  const float inv = 1.f / s;  // a power of two: exact
  for (int h = threadIdx.x; h < H; h += blockDim.x)
    xh[(int64_t)t * H + h] = __float2half_rn(load_as_f32(x, dt, (int64_t)t * H + h) * inv);
  if (threadIdx.x == 0) scale[t] = s;
}

__global__ void __launch_bounds__(kLhThreads, 1) lmhead_gemv_kernel(LmHeadParams p) {
  extern __shared__ __align__(16) unsigned char lh_smem[];
  uint32_t* lut = reinterpret_cast<uint32_t*>(lh_smem);
  __half* xs = reinterpret_cast<__half*>(lh_smem + kLutBytes);
  const int xs_bytes = p.xs_bytes;
  build_lut(lut, p.code, p.code);
  const int n16 = p.T * p.H / 8;
  for (int i = threadIdx.x; i < n16; i += blockDim.x)
    reinterpret_cast<uint4*>(xs)[i] = ldg_u4(p.xh + 8 * (size_t)i);
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const uint32_t ring = smem_u32(lh_smem + kLutBytes + xs_bytes) + warp * kLhStages * kLhStageBytes;
  const uint32_t lanebase = (uint32_t)lane * 4u;
  const uint32_t xrow = smem_u32(xs) + (uint32_t)(g * p.H + 16 * t) * 2u;
  const bool has_tok = g < p.T;
  const int ngroups = (p.V + kLhRows - 1) / kLhRows;
  const int units = ngroups * p.splits;
  const int nw = gridDim.x * kLhWarps;
  const size_t hq = (size_t)(p.H / 64);  // 64-column chunks per row
  for (int u = blockIdx.x * kLhWarps + warp; u < units; u += nw) {
    const int grp = u / p.splits, sp = u - grp * p.splits;
    const int r0 = grp * kLhRows;
    const int c0 = sp * p.cps;                                   // a multiple of kLhSc
    const int nst = (min(p.nchunks, c0 + p.cps) - c0) / kLhSc;   // stages of this unit
    // stage q = chunks c0 + 4q .. +3.  Each copy instruction moves 4 rows x
    // one 128-byte line; a row's 16-byte granule k is stored at k ^ (row & 7)
    // so that the fragment reads below hit every bank pair once.  An empty
    // group past the end keeps the group count uniform.
    auto issue = [&](int q) {
      if (q < nst) {
        const uint32_t c = (uint32_t)(c0 + kLhSc * q);
        const uint32_t st = ring + (uint32_t)(q % kLhStages) * kLhStageBytes;
        const int gi = lane & 7;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int r = 4 * k + (lane >> 3);
          const size_t row = (size_t)min(r0 + r, p.V - 1);
          cp_async16(st + r * kLhRowBytes + 16 * (gi ^ (r & 7)), p.packed + ((row * p.H + 64u * c) >> 1) + 16 * gi);
        }
        if (p.qbs == 64) {
          if (lane < kLhRows) {
            const size_t row = (size_t)min(r0 + lane, p.V - 1);
            cp_async16(st + kLhRows * kLhRowBytes + 16 * lane, p.absmax + row * hq + c);
          }
        } else {
          const int r = lane & 15;
          const size_t row = (size_t)min(r0 + r, p.V - 1);
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * (lane >> 4) + jj;
            cp_async4(st + kLhRows * kLhRowBytes + 16 * r + 4 * j, p.absmax + (row * p.H + 64u * (c + j)) / p.qbs);
          }
        }
      }
      cp_async_commit();
    };
#pragma unroll
    for (int q = 0; q < kLhStages - 1; ++q) issue(q);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < nst; ++q) {
      cp_async_wait<kLhStages - 2>();
      __syncwarp();
      const uint32_t st = ring + (uint32_t)(q % kLhStages) * kLhStageBytes;
#pragma unroll
      for (int j = 0; j < kLhSc; ++j) {
        // x of token g, columns 64c + 16t .. +16 as 8 half2 (slots g >= T are zero)
        uint4 xa = make_uint4(0, 0, 0, 0), xb = make_uint4(0, 0, 0, 0);
        if (has_tok) {
          const uint32_t xaddr = xrow + (uint32_t)(c0 + kLhSc * q + j) * 128u;
          xa = lds_u4(xaddr);
          xb = lds_u4(xaddr + 16);
        }
        // row g (and g + 8): bytes 32j + 8t .. +8 of the stage's line, granule 2j + t/2
        const uint32_t goff = 16u * (uint32_t)((2 * j + (t >> 1)) ^ g) + 8u * (uint32_t)(t & 1);
        const uint2 wa = lds_u2(st + g * kLhRowBytes + goff);
        const uint2 wb = lds_u2(st + (g + 8) * kLhRowBytes + goff);
        const float ama = lds_f32(st + kLhRows * kLhRowBytes + 16 * g + 4 * j);
        const float amb = lds_f32(st + kLhRows * kLhRowBytes + 16 * (g + 8) + 4 * j);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        // MMA m: bytes 2m and 2m+1 of the lane's 8 (columns 16t + 4m .. +4)
        mma_16816(d, lut_lookup<0, 0>(lut, wa.x, lanebase), lut_lookup<0, 0>(lut, wb.x, lanebase),
                  lut_lookup<1, 0>(lut, wa.x, lanebase), lut_lookup<1, 0>(lut, wb.x, lanebase), xa.x, xa.y);
        mma_16816(d, lut_lookup<2, 0>(lut, wa.x, lanebase), lut_lookup<2, 0>(lut, wb.x, lanebase),
                  lut_lookup<3, 0>(lut, wa.x, lanebase), lut_lookup<3, 0>(lut, wb.x, lanebase), xa.z, xa.w);
        mma_16816(d, lut_lookup<0, 0>(lut, wa.y, lanebase), lut_lookup<0, 0>(lut, wb.y, lanebase),
                  lut_lookup<1, 0>(lut, wa.y, lanebase), lut_lookup<1, 0>(lut, wb.y, lanebase), xb.x, xb.y);
        mma_16816(d, lut_lookup<2, 0>(lut, wa.y, lanebase), lut_lookup<2, 0>(lut, wb.y, lanebase),
                  lut_lookup<3, 0>(lut, wa.y, lanebase), lut_lookup<3, 0>(lut, wb.y, lanebase), xb.z, xb.w);
        acc[0] = fmaf(ama, d[0], acc[0]);
        acc[1] = fmaf(ama, d[1], acc[1]);
        acc[2] = fmaf(amb, d[2], acc[2]);
        acc[3] = fmaf(amb, d[3], acc[3]);
      }
      __syncwarp();  // every lane is done with stage q before it is refilled
      issue(q + kLhStages - 1);
    }
    cp_async_wait<0>();
    __syncwarp();
    // D fragment: lane (g, t) holds rows g, g+8 for token slots 2t, 2t+1
    const int ra = r0 + g, rb = ra + 8;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int tok = 2 * t + h;
      if (tok < p.T) {
        float* dst = p.part + ((size_t)sp * p.T + tok) * p.V;
        if (ra < p.V) dst[ra] = acc[h];
        if (rb < p.V) dst[rb] = acc[2 + h];
      }
    }
  }
}

__global__ void lmhead_finalize_kernel(const float* part, const float* scale, int splits, int T, int V,
                                       const void* bias, int bias_dt, void* out, int out_dt) {
  const int64_t total = (int64_t)T * V;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int tok = (int)(i / V), v = (int)(i - (int64_t)tok * V);
    float s = 0.f;
    for (int k = 0; k < splits; ++k) s += __ldcg(part + ((int64_t)k * T + tok) * V + v);
    s *= scale[tok];
    if (bias) s += load_as_f32(bias, bias_dt, v);
    store_from_f32(out, out_dt, i, s);
  }
}

struct LmHeadPlan {
  int splits = 1, cps = 1, nchunks = 0;
  size_t xh_off = 0, scale_off = 0, part_off = 0, bytes = 0;
};

LmHeadPlan lmhead_plan(int T, int V, int H, int sm_count) {
  LmHeadPlan pl;
  pl.nchunks = H / 64;
  const int ngroups = (V + kLhRows - 1) / kLhRows;
  const long want = (long)kLhUnitsPerWarp * sm_count * kLhWarps;
  int splits = (int)std::min<long>(pl.nchunks / kLhSc, std::max<long>(1, (want + ngroups - 1) / ngroups));
  pl.cps = (pl.nchunks + splits - 1) / splits;
  pl.cps = (pl.cps + kLhSc - 1) / kLhSc * kLhSc;   // whole ring stages
  pl.splits = (pl.nchunks + pl.cps - 1) / pl.cps;  // every split has >= 1 stage
  pl.xh_off = 0;
  pl.scale_off = align_up((size_t)T * H * 2, 256);
  pl.part_off = pl.scale_off + align_up((size_t)T * 4, 256);
  pl.bytes = pl.part_off + align_up((size_t)pl.splits * T * V * 4, 256);
  return pl;
}

size_t lmhead_smem_bytes(int T, int H) { return (size_t)kLutBytes + align_up((size_t)T * H * 2, 16) + kLhRingBytes; }

}  // namespace
}  // namespace nsm

using namespace nsm;

extern "C" {

size_t nsm_lm_head_workspace_bytes(int32_t tokens, int32_t out_features, int32_t in_features) {
  if (tokens <= 0 || out_features <= 0 || in_features < 256 || in_features % 256) return 0;
  DeviceInfo di;
  if (current_device(&di) != NSM_OK) return 0;
  return lmhead_plan(tokens, out_features, in_features, di.sm_count).bytes;
}

int nsm_lm_head_max_tokens(int32_t in_features) {
  DeviceInfo di;
  if (in_features < 256 || in_features % 256 || current_device(&di) != NSM_OK) return 0;
  const long room = (long)di.max_smem_optin - 4096 - kLutBytes - kLhRingBytes;  // 4 KB: static tables
  return (int)std::max<long>(0, std::min<long>(kLhMaxTokens, room / (2L * in_features)));
}

int nsm_lm_head_nf4(const void* x, int32_t x_dtype, int32_t tokens, const uint8_t* packed, const float* absmax,
                    const float* code, int32_t out_features, int32_t in_features, int32_t quant_block_size,
                    const void* bias, int32_t bias_dtype, void* out, int32_t out_dtype, void* workspace,
                    size_t workspace_bytes, nsm_stream_t stream) {
  auto dtype_ok = [](int d) { return d == NSM_F32 || d == NSM_F16 || d == NSM_BF16; };
  NSM_REQUIRE(dtype_ok(x_dtype) && dtype_ok(out_dtype) && (bias == nullptr || dtype_ok(bias_dtype)),
              NSM_ERR_INVALID_ARG, "bad dtype");
  NSM_REQUIRE(tokens >= 0 && out_features >= 0, NSM_ERR_INVALID_ARG, "negative size");
  if (tokens == 0 || out_features == 0) return NSM_OK;
  NSM_REQUIRE(in_features >= 256 && in_features % 256 == 0, NSM_ERR_UNSUPPORTED,
              "in_features must be a positive multiple of 256");
  NSM_REQUIRE(quant_block_size >= 64 && quant_block_size % 64 == 0, NSM_ERR_UNSUPPORTED,
              "quant_block_size must be a multiple of 64");
  NSM_REQUIRE((int64_t)out_features * in_features < ((int64_t)1 << 40), NSM_ERR_UNSUPPORTED, "weight too large");
  NSM_REQUIRE(x && packed && absmax && code && out && workspace, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(((uintptr_t)packed & 15) == 0 && ((uintptr_t)absmax & (quant_block_size == 64 ? 15 : 3)) == 0 &&
                  ((uintptr_t)workspace & 255) == 0,
              NSM_ERR_INVALID_ARG,
              "packed must be 16-byte, absmax 16-byte (4-byte unless quant_block_size is 64), workspace 256-byte "
              "aligned");
  DeviceInfo di;
  int st = current_device(&di);
  if (st != NSM_OK) return st;
  NSM_REQUIRE(tokens <= nsm_lm_head_max_tokens(in_features), NSM_ERR_UNSUPPORTED,
              "too many tokens for one call at this in_features (see nsm_lm_head_max_tokens)");
  const LmHeadPlan pl = lmhead_plan(tokens, out_features, in_features, di.sm_count);
  NSM_REQUIRE(workspace_bytes >= pl.bytes, NSM_ERR_WORKSPACE, "workspace too small (nsm_lm_head_workspace_bytes)");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto* ws = static_cast<unsigned char*>(workspace);
  __half* xh = reinterpret_cast<__half*>(ws + pl.xh_off);
  float* scale = reinterpret_cast<float*>(ws + pl.scale_off);
  float* part = reinterpret_cast<float*>(ws + pl.part_off);
  lmhead_prep_kernel<<<tokens, 1024, 0, s>>>(x, x_dtype, in_features, xh, scale);
  NSM_CHECK_CUDA(cudaGetLastError());
  const size_t smem = lmhead_smem_bytes(tokens, in_features);
  {
    // largest dynamic shared memory set so far per device; host threads that
    // call concurrently serialise on the lock
    static std::mutex smem_mu;
    static size_t smem_set[64] = {};
    std::lock_guard<std::mutex> lk(smem_mu);
    const int dslot = di.device & 63;
    if (smem > smem_set[dslot]) {
      NSM_CHECK_CUDA(cudaFuncSetAttribute(lmhead_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      smem_set[dslot] = smem;
    }
  }
  LmHeadParams p;
  p.xh = xh;
  p.packed = packed;
  p.absmax = absmax;
  p.code = code;
  p.part = part;
  p.xs_bytes = (int)align_up((size_t)tokens * in_features * 2, 16);
  p.T = tokens;
  p.V = out_features;
  p.H = in_features;
  p.qbs = quant_block_size;
  p.splits = pl.splits;
  p.cps = pl.cps;
  p.nchunks = pl.nchunks;
  lmhead_gemv_kernel<<<di.sm_count, kLhThreads, smem, s>>>(p);
  NSM_CHECK_CUDA(cudaGetLastError());
  const int64_t total = (int64_t)tokens * out_features;
  const int fgrid = (int)std::min<int64_t>((total + 255) / 256, 8L * di.sm_count);
  lmhead_finalize_kernel<<<fgrid, 256, 0, s>>>(part, scale, pl.splits, tokens, out_features, bias, bias_dtype, out,
                                               out_dtype);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

}  // extern "C"
