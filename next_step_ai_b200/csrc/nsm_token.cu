// nsm_token.cu -- one decode token through a whole stack of sparse-MLP layers
// in ONE persistent kernel (cooperative launch: one 16-warp CTA per SM, all
// co-resident).
//
// Per layer (reference: the per-layer tail of forward_token,
// streaming_llama_runtime.py:7762-7775; routing :4209-4238 / :4311-4352; the
// MLP :5433-5492), phases that the per-layer path runs as separate kernels:
//   A  (the CTAs owning 128-column slices) the previous layer's output: the
//      fixed-order sum of its down partials (and, with several GPUs, the
//      rank-ordered sum over NVLink through the exchange buffers); residual
//      update; RMSNorm weight; x as fp16 hi + lo parts with one power-of-two
//      scale per 64 columns; the slice's partial latent x . enc_w^T and sum
//      of squares;
//   B  (every CTA) the partial latents reduced in a fixed order (identical
//      bits on every CTA), the norm scale, enc_b, the basis top-k mask, and
//      the scores of this CTA's share of the blocks; meanwhile bulk copies
//      bring the whole layer input x into shared memory;
//   C  (every CTA, the same result) exact top-k of the scores (ties to the
//      lower block id) and the selected blocks present in this rank's pool in
//      block-id order;
//   gate/up: every warp streams an equal contiguous range of the (block,
//      64-column tile) pairs with direct 16-byte loads (no shared-memory
//      ring), dequantises through the per-lane lookup table and multiplies on
//      the tensor pipe (mma.sync, fp32 accumulation); a warp flushes fp32
//      partials per block segment; the warp that flushes a block's last
//      segment (atomic ticket) later sums the block's segments in fixed order
//      and publishes SiLU(gate)*up as fp16 hi + lo with a power-of-two scale;
//   down: once every block's activation is published, the CTA stages them in
//      shared memory and every warp streams an equal range of the (64-row
//      group, block) pairs; its fp32 partials per row group are the layer's
//      output, summed by the next layer's phase A.
// Phases are linked by monotonic arrival counters in the workspace
// (release adds, acquire polls, every poll bounded: a wait that runs out
// records NSM_ERR_TIMEOUT in the error word and the CTA leaves the token;
// the others see the error and leave too).  No phase waits on a CTA that is
// still waiting on it, and the cooperative launch guarantees every CTA is
// resident.  The next layer's router slices are prefetched into shared memory
// with bulk copies while the current layer's down projection streams.
//
// Precision of the tensor-core dot products: x and SiLU*up are each split into
// fp16 hi + lo parts carried in columns 0 and 1 of the MMA's 8-column B
// operand (lanes with odd g load the lo part), so one MMA yields both partial
// dot products and their sum carries ~22 bits of the activation; the
// codebook enters the lookup table as fp16(alpha * code) with alpha in [1, 2)
// chosen per codebook to minimise the fp16 rounding of its 16 values, and
// 1/alpha is folded into the fp32 absmax scale.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstring>
#include <mutex>
#include <vector>

#include "nsm_common.cuh"
#include "nsm_internal.h"
#include "nsm_nf4.cuh"
#include "nsm_select.cuh"

namespace nsm {

constexpr int kTkWarps = 8;
constexpr int kTkThreads = kTkWarps * 32;
static_assert(kTkThreads >= 256 && kTkThreads % 128 == 0, "the phases assume 2 to 8 groups of 128 threads");
constexpr int kTkCols = 128;          // phase-A columns per CTA
constexpr int kTkRank = 64;           // router rank of this path
constexpr int kTkMaxK = 256;          // selected blocks per layer
constexpr int kTkMaxNB = 4096;        // router blocks
constexpr int kTkMaxH = 16384;
constexpr int kTkMaxScoreRows = 32;   // blocks scored per CTA (NB <= 32 * gridDim)
constexpr int kTkDepthGU = 2;         // gate/up tile pairs in flight per warp (beyond the one computed)
constexpr int kTkDepthDn = 3;         // down pairs in flight per warp

// ---- device descriptor of one layer (an array of these lives in the workspace)
struct TkLayer {
  const void* enc_w;    // [64][H] bf16 / f16
  const void* enc_b;    // [64] or null
  const void* score_w;  // [NB][64]
  const void* score_b;  // [NB] or null
  const float* dbn;     // [NB] or null
  const void* norm_w;   // [H] or null
  const uint8_t* gate;
  const float* gate_am;
  const uint8_t* up;
  const float* up_am;
  const uint8_t* down;
  const float* down_am;
  const float* gate_code;
  const float* up_code;
  const float* down_code;
  const int32_t* slot_of_block;
  int64_t gstride, gastride, dbs, dabs;  // bytes / floats between pool rows
  int wdtype, norm_dtype, top_k, basis_top_k, legacy, pool_rows, block_begin, block_end;
};

// ---- workspace (caller-owned, zero-filled once)
// The error word sits at byte 8, where the per-layer decode workspace keeps
// its own, so nsm_workspace_error reads either kind of workspace.
struct TkSync {
  unsigned y_done, a_done;
  int err;
  unsigned b_done, act_done, exit_count;
  unsigned long long* stamps;  // optional phase timestamps (nsm_token_profile)
  int stamp_layers;
  unsigned pad[5];
};
static_assert(offsetof(TkSync, err) == 8, "error word offset");
constexpr int kTkStamps = 8;  // per CTA and layer: A in, A out, B in, B out, C out, gate/up out, act in, down out

struct TkWs {
  TkSync* sync;
  TkLayer* layers;
  float* ypart;        // [kMaxSlotGroups][H]
  float* latent_part;  // [H/128][64]
  float* sumsq_part;   // [H/128]
  float* scores;       // [NB]
  __half* x_hi;        // [H]
  __half* x_lo;        // [H]
  float* xscale;       // [H/64] (+ padding to 16 bytes)
  float* gu_part;      // [kTkMaxK][kMaxUnitsPerSlot][64]
  unsigned* ticket;    // [kTkMaxK]
  __half* act_hi;      // [kTkMaxK][32]
  __half* act_lo;      // [kTkMaxK][32]
  float* act_scale;    // [kTkMaxK]
  size_t bytes;
};

static TkWs tk_ws_layout(void* base, int H, int NB, int L) {
  TkWs w{};
  char* b = reinterpret_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = b ? b + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  w.sync = reinterpret_cast<TkSync*>(take(sizeof(TkSync)));
  w.layers = reinterpret_cast<TkLayer*>(take((size_t)std::max(L, 1) * sizeof(TkLayer)));
  w.ypart = reinterpret_cast<float*>(take((size_t)kMaxSlotGroups * H * sizeof(float)));
  w.latent_part = reinterpret_cast<float*>(take((size_t)(H / kTkCols) * kTkRank * sizeof(float)));
  w.sumsq_part = reinterpret_cast<float*>(take((size_t)(H / kTkCols) * sizeof(float)));
  w.scores = reinterpret_cast<float*>(take((size_t)NB * sizeof(float)));
  w.x_hi = reinterpret_cast<__half*>(take((size_t)H * sizeof(__half)));
  w.x_lo = reinterpret_cast<__half*>(take((size_t)H * sizeof(__half)));
  w.xscale = reinterpret_cast<float*>(take((size_t)(H / 64) * sizeof(float) + 16));
  w.gu_part = reinterpret_cast<float*>(take((size_t)kTkMaxK * kMaxUnitsPerSlot * 64 * sizeof(float)));
  w.ticket = reinterpret_cast<unsigned*>(take((size_t)kTkMaxK * sizeof(unsigned)));
  w.act_hi = reinterpret_cast<__half*>(take((size_t)kTkMaxK * 32 * sizeof(__half)));
  w.act_lo = reinterpret_cast<__half*>(take((size_t)kTkMaxK * 32 * sizeof(__half)));
  w.act_scale = reinterpret_cast<float*>(take((size_t)kTkMaxK * sizeof(float)));
  w.bytes = off;
  return w;
}

struct TkParams {
  TkWs ws;
  float* residual;
  int H, NB, L;
  float eps;
  ExchangeDev ex;
  int wait_spins;         // bound of one counter / mbarrier wait (polls)
  int* trace_blocks;      // [L][trace_k] or null
  int* trace_counts;      // [L] or null
  float* trace_residual;  // [L][H] or null
  int trace_k;            // row stride of trace_blocks
};

// ---- shared-memory layout (bytes from the dynamic base, which sits at 0x400)
constexpr int kTkLutOff = 0;                                    // 2 tables, 64 KB
constexpr int kTkLutScratch = kLutBytes;                        // 2 KB pair scratch
constexpr int kTkXOff = kLutBytes + 2048;                       // x hi | x lo | xscale  (act overlays)
constexpr int kTkXBytes = kTkMaxH * 2 * 2 + (kTkMaxH / 64) * 4 + 16;
constexpr int kTkEncOff = (kTkXOff + kTkXBytes + 127) / 128 * 128;  // [64][128] 2-byte
constexpr int kTkSrowOff = kTkEncOff + kTkRank * kTkCols * 2;   // [32][64] 2-byte score rows
constexpr int kTkGammaOff = kTkSrowOff + kTkMaxScoreRows * kTkRank * 2;  // [128] raw (<= 512 B)
constexpr int kTkKeyOff = kTkGammaOff + kTkCols * 4;            // [NB] u32
constexpr int kTkSelOff = kTkKeyOff + kTkMaxNB * 4;             // RadixSelectSmem
constexpr int kTkRowsOff = kTkSelOff + 2560;                    // [k] pool rows
constexpr int kTkMiscOff = kTkRowsOff + kTkMaxK * 4;            // per-CTA state
constexpr int kTkBarOff = kTkMiscOff + 4096;                    // mbarriers: router prefetch, x staging
constexpr int kTkSmem = kTkBarOff + 64;
static_assert(sizeof(RadixSelectSmem) <= 2560, "selection scratch");
static_assert(kTkSmem <= 227 * 1024, "token kernel shared memory");
static_assert(kTkXOff % 1024 == 0 && kTkEncOff % 16 == 0 && kTkSrowOff % 16 == 0 && kTkGammaOff % 16 == 0,
              "alignment");
// act overlay inside the x region: hi [k][32] | lo [k][32] | scale [k]
static_assert(kTkMaxK * 32 * 2 * 2 + kTkMaxK * 4 <= kTkXBytes, "act overlay");
static_assert(kTkRank * kTkCols * 2 >= 4096 * 4 && kTkMaxScoreRows * kTkRank * 2 >= 1024 * 4,
              "selection scratch in the consumed router buffers");

// per-CTA state in the misc region
struct TkMisc {
  float latent[kTkRank];
  float xs[kTkCols];
  float ysum[4][kTkCols];
  float red[32];
  float inv_alpha[2];   // 1 / alpha of LUT tables 0 (gate) and 1 (up)
  float code_cur[3][16];
  int down_table;       // LUT table of the down code (0 or 1)
  float norm_scale;
  int count_prev;       // selected blocks of the previous layer (its down output is pending)
  int abort;
  unsigned act_target;  // running act_done target
  uint32_t bar_phase;   // parity of the router prefetch mbarrier
  int pf_out;           // a router prefetch is in flight
  int layer;            // the layer being decoded
  uint32_t x_phase;     // parity of the x staging mbarrier
  int x_out;            // an x staging copy is in flight
};
static_assert(sizeof(TkMisc) <= 4096, "misc region");

__device__ __forceinline__ char* tk_smem() { return reinterpret_cast<char*>(g_lut_smem); }
__device__ __forceinline__ TkMisc& tk_misc() { return *reinterpret_cast<TkMisc*>(tk_smem() + kTkMiscOff); }
__device__ __forceinline__ unsigned long long tk_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- inter-CTA synchronisation ------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) {
  int v;
  asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void tk_fail(const TkParams& p, int code) {
  atomicCAS(&p.ws.sync->err, 0, code);
  tk_misc().abort = 1;
}
constexpr unsigned kTkPollSleepNs = 256;
// CTA-wide wait until *ctr has reached `target` (wrap-safe).  Thread 0 polls
// with acquire loads, at most p.wait_spins times; a wait that runs out, or an
// error another CTA recorded, makes the CTA leave the token.  Returns false
// then.  Every thread of the CTA must call it.
__device__ bool tk_wait(const TkParams& p, const unsigned* ctr, unsigned target) {
  TkMisc& M = tk_misc();
  if (threadIdx.x == 0 && !M.abort) {
    // polls back off (up to kTkPollSleepNs between reads) so that CTAs waiting on
    // a counter do not hammer its L2 line while the others still stream
    unsigned ns = 32;
    for (int it = 0;; ++it) {
      if ((int)(ld_acquire_u32(ctr) - target) >= 0) break;
      if (it >= p.wait_spins) {
        tk_fail(p, NSM_ERR_TIMEOUT);
        break;
      }
      if ((it & 15) == 15 && ld_volatile_i32(&p.ws.sync->err) != 0) {
        M.abort = 1;
        break;
      }
      __nanosleep(ns);
      ns = min(ns * 2u, kTkPollSleepNs);
    }
  }
  __syncthreads();
  return !M.abort;
}
// Every thread's earlier global writes, then one release add by thread 0.
__device__ __forceinline__ void tk_arrive(unsigned* ctr) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) red_release_add(ctr, 1u);
}

// ---- lookup table with the prescaled codebooks -------------------------------------
// Table t (0: gate, 1: up) holds half2 {fp16(a_t * code[hi]), fp16(a_t * code[lo])}
// per packed byte; a_t in [1, 2) minimises sum_k (fp16(a * c_k) / a - c_k)^2 over
// 256 candidates (ties to the smaller a); 1 / a_t goes into the absmax scale.
// The down code must equal one of the two by value (the LUT serves it too).
__device__ __noinline__ void tk_build_lut(const TkParams& p, const TkLayer& L) {
  TkMisc& M = tk_misc();
  char* sm = tk_smem();
  float* errs = reinterpret_cast<float*>(sm + kTkKeyOff);  // [2][256] + 2 (the keys are free here)
  uint32_t* pairs = reinterpret_cast<uint32_t*>(sm + kTkLutScratch);
  const int tid = threadIdx.x;
  if (tid < 48) M.code_cur[tid >> 4][tid & 15] = (tid < 16 ? L.gate_code : tid < 32 ? L.up_code : L.down_code)[tid & 15];
  __syncthreads();
  for (int ti = tid; ti < 512; ti += blockDim.x) {  // two tables x 256 candidates
    const int t = ti >> 8, i = ti & 255;
    const float a = 1.f + (float)i * (1.f / 256.f);
    float e = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float c = M.code_cur[t][k];
      const float h = __half2float(__float2half_rn(a * c));
      const float d = h / a - c;
      e = fmaf(d, d, e);
    }
    errs[t * 256 + i] = e;
  }
  __syncthreads();
  if (tid < 64) {  // warp 0: table 0, warp 1: table 1; lane l scans candidates l, l+32, ...
    const int t = tid >> 5, lane = tid & 31;
    float be = errs[t * 256 + lane];
    int bi = lane;
    for (int i = lane + 32; i < 256; i += 32) {
      const float e = errs[t * 256 + i];
      if (e < be) {
        be = e;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float oe = __shfl_xor_sync(0xffffffffu, be, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oe < be || (oe == be && oi < bi)) {
        be = oe;
        bi = oi;
      }
    }
    if (lane == 0) {
      const float a = 1.f + (float)bi * (1.f / 256.f);
      M.inv_alpha[t] = 1.f / a;
      errs[512 + t] = a;
    }
  }
  __syncthreads();
  for (int i = tid; i < 512; i += blockDim.x) {
    const int t = i >> 8, e = i & 255;
    const float a = errs[512 + t];
    const __half lo = __float2half_rn(a * M.code_cur[t][e >> 4]);
    const __half hi = __float2half_rn(a * M.code_cur[t][e & 15]);
    pairs[i] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
  }
  if (tid == 0) {
    bool eq0 = true, eq1 = true;
    for (int k = 0; k < 16; ++k) {
      eq0 &= M.code_cur[2][k] == M.code_cur[0][k];
      eq1 &= M.code_cur[2][k] == M.code_cur[1][k];
    }
    M.down_table = eq0 ? 0 : 1;
    if (!eq0 && !eq1) tk_fail(p, NSM_ERR_UNSUPPORTED);
  }
  __syncthreads();
  uint4* lut4 = reinterpret_cast<uint4*>(sm + kTkLutOff);
  for (int i = tid; i < 256 * kLutWordsPerEntry / 4; i += blockDim.x) {
    const uint32_t v = pairs[((i >> 3) & 1) * 256 + (i >> 4)];
    lut4[i] = make_uint4(v, v, v, v);
  }
  __syncthreads();
}

// true (every thread) when the layer's codebooks are the ones the LUT holds
__device__ __noinline__ bool tk_codes_match(const TkLayer& L) {
  TkMisc& M = tk_misc();
  int diff = 0;
  if (threadIdx.x < 48) {
    const int t = threadIdx.x >> 4, k = threadIdx.x & 15;
    const float v = (t == 0 ? L.gate_code : t == 1 ? L.up_code : L.down_code)[k];
    diff = v != M.code_cur[t][k];
  }
  return __syncthreads_or(diff) == 0;
}

// ---- bulk copies into shared memory -------------------------------------------------
__device__ __forceinline__ void tk_bulk(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ uint32_t align16_dev(uint32_t v) { return (v + 15u) & ~15u; }
__device__ __forceinline__ int tk_score_lo(int NB, int cta) { return (int)(((long long)NB * cta) / gridDim.x); }

// This CTA's slices of layer L's router weights (encoder columns, RMSNorm
// weight, score-head rows).  Called by warp 0 (every lane) once nothing reads
// the buffers any more.
__device__ __forceinline__ void tk_prefetch_router(const TkParams& p, const TkLayer& L) {
  char* sm = tk_smem();
  const int lane = threadIdx.x & 31, cta = blockIdx.x;
  const uint32_t bar = smem_u32(sm + kTkBarOff);
  const bool colslice = cta < p.H / kTkCols;
  const int b0 = tk_score_lo(p.NB, cta), b1 = tk_score_lo(p.NB, cta + 1);
  const int esz = L.norm_dtype == NSM_F32 ? 4 : 2;
  uint32_t bytes = (uint32_t)(b1 - b0) * kTkRank * 2;
  if (colslice) bytes += kTkRank * kTkCols * 2 + (L.norm_w ? kTkCols * esz : 0);
  if (lane == 0) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, bytes);
  }
  __syncwarp();
  if (colslice) {
    const int c0 = cta * kTkCols;
    const char* enc = reinterpret_cast<const char*>(L.enc_w);
    for (int r = lane; r < kTkRank; r += 32)
      tk_bulk(smem_u32(sm + kTkEncOff + r * kTkCols * 2), enc + ((int64_t)r * p.H + c0) * 2, kTkCols * 2, bar);
    if (lane == 0 && L.norm_w)
      tk_bulk(smem_u32(sm + kTkGammaOff), reinterpret_cast<const char*>(L.norm_w) + (int64_t)c0 * esz, kTkCols * esz,
              bar);
  }
  if (lane == 1 && b1 > b0)
    tk_bulk(smem_u32(sm + kTkSrowOff), reinterpret_cast<const char*>(L.score_w) + (int64_t)b0 * kTkRank * 2,
            (uint32_t)(b1 - b0) * kTkRank * 2, bar);
}
// CTA-wide bounded wait for the router prefetch of the current layer.
__device__ bool tk_wait_router(const TkParams& p) {
  TkMisc& M = tk_misc();
  if (threadIdx.x == 0 && !M.abort)
    if (!mbar_wait(smem_u32(tk_smem() + kTkBarOff), M.bar_phase, p.wait_spins)) tk_fail(p, NSM_ERR_TIMEOUT);
  __syncthreads();
  return !M.abort;
}

// Thread 0, after the wait on phase A: the layer input (x hi, lo, scales) into the
// shared-memory x region with bulk copies, which land while phase B and the
// selection run.  x was written by other CTAs through the generic proxy; the
// acquire of their arrivals plus a proxy fence order those writes before the
// async-proxy reads.
__device__ __forceinline__ void tk_issue_x(const TkParams& p, uint32_t xbar) {
  char* sm = tk_smem();
  TkMisc& M = tk_misc();
  const uint32_t xb = (uint32_t)p.H * 2u;
  const uint32_t sb = align16_dev((uint32_t)(p.H / 64) * 4u);
  asm volatile("fence.proxy.async.global;" ::: "memory");
  fence_proxy_async_smem();
  mbar_arrive_expect_tx(xbar, 2u * xb + sb);
  const uint32_t dst = smem_u32(sm + kTkXOff);
  tk_bulk(dst, p.ws.x_hi, xb, xbar);
  tk_bulk(dst + xb, p.ws.x_lo, xb, xbar);
  tk_bulk(dst + 2u * xb, p.ws.xscale, sb, xbar);
  M.x_out = 1;
}

__device__ __forceinline__ float tk_load(const void* ptr, int dtype, int64_t i) { return load_as_f32(ptr, dtype, i); }
__device__ __forceinline__ float tk_from16(uint16_t v, int wdtype) {
  return wdtype == NSM_F16 ? __half2float(__ushort_as_half(v)) : __uint_as_float((uint32_t)v << 16);
}

// ---- the previous layer's output for this CTA's 128 columns -----------------------
// Fixed-order sum of the down segments of each column (4 quarter sums, then
// combined in order); with several GPUs the rank-ordered sum over NVLink.
// Result in M.xs (threads < 128 hold their column).  Returns false on abort.
__device__ __noinline__ bool tk_pending_output(const TkParams& p, int c0, int cnt, uint32_t epoch) {
  TkMisc& M = tk_misc();
  const int tid = threadIdx.x, col = tid & (kTkCols - 1);
  int nseg = 0;
  if (cnt > 0) {
    const int RP = p.H >> 6, total = RP * cnt;
    const int nwd = stream_warps(RP, cnt, kMaxSlotGroups, (int)gridDim.x * kTkWarps);
    const int rg = (c0 + col) >> 6;
    nseg = stream_owner(total, nwd, rg * cnt + cnt - 1) - stream_owner(total, nwd, rg * cnt) + 1;
  }
  // quarter q sums segments q, q + 4, q + 8, ... of the column
  for (int q = tid / kTkCols; q < 4; q += kTkThreads / kTkCols) {
    float y = 0.f;
    float v[kMaxSlotGroups / 4];
#pragma unroll
    for (int u = 0; u < kMaxSlotGroups / 4; ++u) {
      const int sg = q + 4 * u;
      v[u] = sg < nseg ? ldcg_f32(p.ws.ypart + (int64_t)sg * p.H + c0 + col) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kMaxSlotGroups / 4; ++u) y += v[u];
    M.ysum[q][col] = y;
  }
  __syncthreads();
  float y = 0.f;
  bool timed_out = false;
  if (tid < kTkCols) {
    y = (M.ysum[0][tid] + M.ysum[1][tid]) + (M.ysum[2][tid] + M.ysum[3][tid]);
    const ExchangeDev& ex = p.ex;
    if (ex.world > 1) {
      const int slot = (int)(epoch & 1u);
      const unsigned long long word = (unsigned long long)__float_as_uint(y) | ((unsigned long long)epoch << 32);
      for (int r = 0; r < ex.world; ++r)
        st_relaxed_sys_u64(ex.data[r] + ((int64_t)slot * ex.world + ex.rank) * ex.hidden + c0 + tid, word);
      const unsigned long long* src = ex.data[ex.rank] + (int64_t)slot * ex.world * ex.hidden + c0 + tid;
      float sum = 0.f;
      for (int r = 0; r < ex.world; ++r) {
        const unsigned long long* w = src + (int64_t)r * ex.hidden;
        unsigned long long v = ld_relaxed_sys_u64(w);
        for (int it = 0; (uint32_t)(v >> 32) != epoch; ++it) {
          if (it >= ex.spin_limit) {
            timed_out = true;
            break;
          }
          v = ld_relaxed_sys_u64(w);
        }
        sum += __uint_as_float((uint32_t)v);
      }
      y = sum;
    }
    M.xs[tid] = y;
  }
  if (__syncthreads_or(timed_out)) {
    if (tid == 0) tk_fail(p, NSM_ERR_TIMEOUT);
    __syncthreads();
    return false;
  }
  return true;
}

// ---- phase A: residual, RMSNorm weight, x hi/lo, partial latent --------------------
__device__ __noinline__ void tk_phase_a(const TkParams& p, const TkLayer& L, int l, int c0, bool pending,
                                        int cnt_prev, uint32_t epoch) {
  TkMisc& M = tk_misc();
  char* sm = tk_smem();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, cta = blockIdx.x;
  if (pending) {
    if (!tk_pending_output(p, c0, cnt_prev, epoch)) return;
  } else {
    if (tid < kTkCols) M.xs[tid] = 0.f;
    __syncthreads();
  }
  float sq = 0.f;
  if (tid < kTkCols) {
    const int c = c0 + tid;
    const float r = p.residual[c] + M.xs[tid];
    if (pending) p.residual[c] = r;
    if (p.trace_residual) p.trace_residual[(int64_t)l * p.H + c] = r;
    sq = r * r;
    float gmul = 1.f;
    if (L.norm_w) {
      const char* gsm = sm + kTkGammaOff;
      gmul = L.norm_dtype == NSM_F32 ? reinterpret_cast<const float*>(gsm)[tid]
                                     : tk_from16(reinterpret_cast<const uint16_t*>(gsm)[tid], L.norm_dtype);
    }
    M.xs[tid] = r * gmul;
  }
  sq = warp_sum(sq);
  if (lane == 0 && warp < kTkCols / 32) M.red[warp] = sq;
  __syncthreads();
  // x as fp16 hi + lo with one power-of-two scale per 64 columns (warps 0, 1)
  if (warp < kTkCols / 64) {
    const float a = M.xs[warp * 64 + lane], b = M.xs[warp * 64 + 32 + lane];
    const float sc = pow2_scale_for(warp_max(fmaxf(fabsf(a), fabsf(b))));
    const float inv = 1.f / sc;
    const int c = c0 + warp * 64;
    const __half ah = __float2half_rn(a * inv), bh = __float2half_rn(b * inv);
    p.ws.x_hi[c + lane] = ah;
    p.ws.x_hi[c + 32 + lane] = bh;
    p.ws.x_lo[c + lane] = __float2half_rn(a * inv - __half2float(ah));
    p.ws.x_lo[c + 32 + lane] = __float2half_rn(b * inv - __half2float(bh));
    if (lane == 0) p.ws.xscale[c >> 6] = sc;
  }
  // partial latent: thread (rank r, eighth e) over 16 columns, reduced over e
  // (a warp holds 4 whole ranks, so every lane of a warp takes the same turns)
  for (int r = tid >> 3; r < kTkRank; r += kTkThreads / 8) {
    const int e = tid & 7;
    const uint4* row = reinterpret_cast<const uint4*>(sm + kTkEncOff + r * kTkCols * 2 + e * 32);
    const uint4 w0 = row[0], w1 = row[1];
    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float lo = tk_from16((uint16_t)(w[i] & 0xffffu), L.wdtype);
      const float hi = tk_from16((uint16_t)(w[i] >> 16), L.wdtype);
      acc = fmaf(lo, M.xs[e * 16 + 2 * i], acc);
      acc = fmaf(hi, M.xs[e * 16 + 2 * i + 1], acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    if (e == 0) p.ws.latent_part[cta * kTkRank + r] = acc;
  }
  if (tid == 0) p.ws.sumsq_part[cta] = (M.red[0] + M.red[1]) + (M.red[2] + M.red[3]);
}

// ---- phase B: latent, norm scale, this CTA's block scores -------------------------
__device__ __noinline__ void tk_phase_b(const TkParams& p, const TkLayer& L) {
  TkMisc& M = tk_misc();
  char* sm = tk_smem();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nA = p.H / kTkCols;
  float* grp = reinterpret_cast<float*>(sm + kTkKeyOff);  // [32][64] (the keys region is free here)
  for (int g = tid >> 4; g < 32; g += kTkThreads / 16) {  // 32 groups of partials
    const int c4 = tid & 15;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4* base = reinterpret_cast<const float4*>(p.ws.latent_part) + c4;
    float4 v[4];
    for (int b0 = g; b0 < nA; b0 += 128) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int b = b0 + 32 * u;
        v[u] = b < nA ? __ldcg(base + b * (kTkRank / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a.x += v[u].x;
        a.y += v[u].y;
        a.z += v[u].z;
        a.w += v[u].w;
      }
    }
    grp[g * kTkRank + 4 * c4 + 0] = a.x;
    grp[g * kTkRank + 4 * c4 + 1] = a.y;
    grp[g * kTkRank + 4 * c4 + 2] = a.z;
    grp[g * kTkRank + 4 * c4 + 3] = a.w;
  }
  if (warp == 2) {
    float t = 0.f;
    for (int b = lane; b < nA; b += 32) t += ldcg_f32(p.ws.sumsq_part + b);
    t = warp_sum(t);
    if (lane == 0) M.norm_scale = 1.f / sqrtf(t / (float)p.H + p.eps);
  }
  __syncthreads();
  if (tid < kTkRank) {
    float acc = 0.f;
    for (int g = 0; g < 32; ++g) acc += grp[g * kTkRank + tid];
    acc *= M.norm_scale;
    if (L.enc_b) acc += tk_load(L.enc_b, L.wdtype, tid);
    M.latent[tid] = acc;
  }
  __syncthreads();
  const int bk = max(1, min(L.basis_top_k, kTkRank));
  if (bk < kTkRank) {
    float keep = 0.f;
    if (tid < kTkRank) {
      const float a = fabsf(M.latent[tid]);
      int pos = 0;
      for (int q = 0; q < kTkRank; ++q) {
        const float b = fabsf(M.latent[q]);
        pos += (b > a) || (b == a && q < tid);
      }
      keep = pos < bk ? M.latent[tid] : 0.f;
    }
    __syncthreads();
    if (tid < kTkRank) M.latent[tid] = keep;
    __syncthreads();
  }
  // scores of blocks [b0, b1): one warp per block, lanes over ranks r and r + 32
  const int b0 = tk_score_lo(p.NB, blockIdx.x), b1 = tk_score_lo(p.NB, blockIdx.x + 1);
  const uint16_t* srow = reinterpret_cast<const uint16_t*>(sm + kTkSrowOff);
  for (int b = b0 + warp; b < b1; b += kTkWarps) {
    const uint16_t* row = srow + (b - b0) * kTkRank;
    const float w0 = tk_from16(row[lane], L.wdtype), w1 = tk_from16(row[lane + 32], L.wdtype);
    float l0 = M.latent[lane], l1 = M.latent[lane + 32];
    if (L.legacy) {
      l0 = fabsf(l0);
      l1 = fabsf(l1);
    }
    float acc = warp_sum(fmaf(l0, w0, l1 * w1));
    if (!L.legacy) {
      if (L.score_b) acc += tk_load(L.score_b, L.wdtype, b);
      acc = fmaxf(acc, 0.f);
    }
    if (L.dbn) acc *= __ldg(L.dbn + b);
    if (lane == 0) p.ws.scores[b] = acc;
  }
}

__device__ __forceinline__ int tk_map_block(const TkLayer& L, int b) {
  int r;
  if (L.slot_of_block != nullptr) r = __ldg(L.slot_of_block + b);
  else r = (b >= L.block_begin && b < L.block_end) ? b - L.block_begin : -1;
  return (r >= 0 && r < L.pool_rows) ? r : -1;
}

// ---- exact k-th largest key in one histogram pass ----------------------------------
// 4096 bins on the top 12 bits of the order-preserving keys (sign, exponent and
// three mantissa bits of the score); a block scan from the top finds the bin
// holding the k-th largest key, and the keys of that bin are ranked pairwise
// (larger key first, ties to the lower index).  Out: the k-th largest key
// *thr, how many of the keys equal to it are selected (*take_eq, the lowest
// indices) and how many there are (*n_thr).  Returns false (nothing written)
// when the bin holds more than kTkRankMax keys.
constexpr int kTkRankMax = 1024;
__device__ bool tk_select_hist(const uint32_t* keys, int NB, int k, uint32_t* thr_out, int* take_out, int* neq_out) {
  char* sm = tk_smem();
  int* hist = reinterpret_cast<int*>(sm + kTkEncOff);    // [4096] (the encoder slice is consumed)
  int* list = reinterpret_cast<int*>(sm + kTkSrowOff);   // [kTkRankMax] (the score rows are consumed)
  RadixSelectSmem& S = *reinterpret_cast<RadixSelectSmem*>(sm + kTkSelOff);
  const int tid = threadIdx.x;
  for (int i = tid; i < 4096; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < NB; i += blockDim.x) atomicAdd(&hist[keys[i] >> 20], 1);
  __syncthreads();
  // thread t owns bins 4095 - kPer t ... 4096 - kPer (t + 1) (descending)
  constexpr int kPer = (4096 + kTkThreads - 1) / kTkThreads;
  int c[kPer], loc = 0;
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    const int b = 4095 - kPer * tid - e;
    c[e] = b >= 0 ? hist[b] : 0;
    loc += c[e];
  }
  int tot;
  const int excl = block_exclusive_scan_s(loc, &tot, S.wsum);
  if (excl < k && k <= excl + loc) {
    int run = excl;
#pragma unroll
    for (int e = 0; e < kPer; ++e) {
      if (run < k && k <= run + c[e]) {
        S.start = 4095 - kPer * tid - e;  // the threshold bin
        S.need = k - run;              // keys to take from it
        S.bin_count = c[e];
      }
      run += c[e];
    }
  }
  __syncthreads();
  const int bin = S.start, need = S.need, m = S.bin_count;
  if (m > kTkRankMax) return false;  // uniform
  // the bin's key indices, in index order
  const int per = (NB + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = min(NB, tid * per), hi = min(NB, lo + per);
  int mine = 0;
  for (int i = lo; i < hi; ++i) mine += (int)(keys[i] >> 20) == bin;
  int pos = block_exclusive_scan_s(mine, &tot, S.wsum);
  for (int i = lo; i < hi; ++i)
    if ((int)(keys[i] >> 20) == bin) list[pos++] = i;
  __syncthreads();
  // rank need - 1 is the k-th largest key (ranks are unique)
  for (int e = tid; e < m; e += blockDim.x) {
    const int ie = list[e];
    const uint32_t ke = keys[ie];
    int r = 0;
    for (int f = 0; f < m; ++f) {
      const uint32_t kf = keys[list[f]];
      r += kf > ke || (kf == ke && list[f] < ie);
    }
    if (r == need - 1) S.prefix = ke;
  }
  __syncthreads();
  const uint32_t thr = S.prefix;
  int gt = 0, eq = 0;
  for (int e = tid; e < m; e += blockDim.x) {
    const uint32_t ke = keys[list[e]];
    gt += ke > thr;
    eq += ke == thr;
  }
  int gt_all, eq_all;
  block_exclusive_scan_s(gt, &gt_all, S.wsum);
  block_exclusive_scan_s(eq, &eq_all, S.wsum);
  *thr_out = thr;
  *take_out = need - gt_all;
  *neq_out = eq_all;
  return true;
}

// ---- phase C: exact top-k, the selected blocks present here in block-id order -------
__device__ __noinline__ int tk_phase_c(const TkParams& p, const TkLayer& L, int l) {
  char* sm = tk_smem();
  uint32_t* keys = reinterpret_cast<uint32_t*>(sm + kTkKeyOff);
  RadixSelectSmem& S = *reinterpret_cast<RadixSelectSmem*>(sm + kTkSelOff);
  int* srows = reinterpret_cast<int*>(sm + kTkRowsOff);
  const int tid = threadIdx.x, NB = p.NB;
  const int k = max(1, min(L.top_k, NB));
  uint32_t kor = 0u, kand = 0xffffffffu;
  for (int i0 = 0; i0 < NB; i0 += 8 * (int)blockDim.x) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * (int)blockDim.x + tid;
      v[u] = i < NB ? ldcg_f32(p.ws.scores + i) : 0.f;
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
  __syncthreads();
  uint32_t thr;
  int take_eq, n_thr;
  if (!tk_select_hist(keys, NB, k, &thr, &take_eq, &n_thr)) {
    // the threshold bin of the 12-bit histogram is too crowded to rank pairwise
    block_radix_select(keys, NB, k, kor, kand, S);
    thr = S.prefix;
    take_eq = S.need;
    n_thr = S.bin_count;
  }
  const bool split = take_eq != n_thr;
  const int per = (NB + (int)blockDim.x - 1) / (int)blockDim.x;
  const int lo = min(NB, tid * per), hi = min(NB, lo + per);
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
    m += sel && tk_map_block(L, i) >= 0;
  }
  int pos = block_exclusive_scan_s(m, &tot, S.wsum);
  for (int i = lo, e = eq_before; i < hi; ++i) {
    const uint32_t key = keys[i];
    const bool sel = key > thr || (key == thr && (!split || e++ < take_eq));
    const int r = sel ? tk_map_block(L, i) : -1;
    if (r < 0) continue;
    srows[pos] = r;
    if (blockIdx.x == 0 && p.trace_blocks) p.trace_blocks[(int64_t)l * p.trace_k + pos] = i;
    ++pos;
  }
  if (blockIdx.x == 0 && tid == 0 && p.trace_counts) p.trace_counts[l] = tot;
  __syncthreads();
  return tot;
}

// ---- gate/up: direct-load stream over (block, 64-column tile) pairs -----------------
struct TkTile {
  uint4 w[2][2];  // [proj][row group]: rows 16rg+g (.x .y) and 16rg+g+8 (.z .w), bytes [8t, 8t+8)
  float4 am[2];   // [proj]: absmax of rows g, g+8, 16+g, 24+g
};

template <int kTable>
__device__ __forceinline__ void tk_rowgroup(uint32_t lb, const uint4 w, const uint32_t b[8], float d[4]) {
  mma_16816_z(d, lut_get<0x400>(w.x, lb, 0, kTable), lut_get<0x400>(w.z, lb, 0, kTable),
              lut_get<0x400>(w.x, lb, 1, kTable), lut_get<0x400>(w.z, lb, 1, kTable), b[0], b[1]);
  mma_16816(d, lut_get<0x400>(w.x, lb, 2, kTable), lut_get<0x400>(w.z, lb, 2, kTable),
            lut_get<0x400>(w.x, lb, 3, kTable), lut_get<0x400>(w.z, lb, 3, kTable), b[2], b[3]);
  mma_16816(d, lut_get<0x400>(w.y, lb, 0, kTable), lut_get<0x400>(w.w, lb, 0, kTable),
            lut_get<0x400>(w.y, lb, 1, kTable), lut_get<0x400>(w.w, lb, 1, kTable), b[4], b[5]);
  mma_16816(d, lut_get<0x400>(w.y, lb, 2, kTable), lut_get<0x400>(w.w, lb, 2, kTable),
            lut_get<0x400>(w.y, lb, 3, kTable), lut_get<0x400>(w.w, lb, 3, kTable), b[6], b[7]);
}

// acc[proj][i] += (W_rows . x_tile) * absmax * scale; D columns 2t (hi) and 2t+1 (lo) summed
__device__ __forceinline__ void tk_tile(const TkTile& tl, const uint32_t b[8], float sg, float su, uint32_t lb,
                                        float acc[2][4]) {
  float d[4];
#pragma unroll
  for (int rg = 0; rg < 2; ++rg) {
    tk_rowgroup<0>(lb, tl.w[0][rg], b, d);
    const float g0 = rg ? tl.am[0].z : tl.am[0].x, g1 = rg ? tl.am[0].w : tl.am[0].y;
    acc[0][rg * 2] = fmaf(d[0] + d[1], g0 * sg, acc[0][rg * 2]);
    acc[0][rg * 2 + 1] = fmaf(d[2] + d[3], g1 * sg, acc[0][rg * 2 + 1]);
    tk_rowgroup<1>(lb, tl.w[1][rg], b, d);
    const float u0 = rg ? tl.am[1].z : tl.am[1].x, u1 = rg ? tl.am[1].w : tl.am[1].y;
    acc[1][rg * 2] = fmaf(d[0] + d[1], u0 * su, acc[1][rg * 2]);
    acc[1][rg * 2 + 1] = fmaf(d[2] + d[3], u1 * su, acc[1][rg * 2 + 1]);
  }
}

// The block's gate/up segments (fixed order), RMSNorm scale, SiLU(gate)*up as
// fp16 hi + lo with one power-of-two scale per block; then the block's ticket
// is reset and the activation counter advanced.  Whole warp, lane = neuron.
// total / nw: the gate/up stream's pairs and warps, tpr its tiles per block.
__device__ __noinline__ void tk_act(const TkParams& p, int s, int total, int nw, int tpr) {
  const int lane = threadIdx.x & 31;
  const int nseg = stream_owner(total, nw, s * tpr + tpr - 1) - stream_owner(total, nw, s * tpr) + 1;
  __threadfence();
  const float* base = p.ws.gu_part + (int64_t)s * kMaxUnitsPerSlot * 64;
  float gs = 0.f, us = 0.f;
  for (int j0 = 0; j0 < nseg; j0 += 4) {
    float vg[4], vu[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = j0 + u;
      vg[u] = j < nseg ? ldcg_f32(base + j * 64 + lane) : 0.f;
      vu[u] = j < nseg ? ldcg_f32(base + j * 64 + 32 + lane) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (j0 + u < nseg) {
        gs += vg[u];
        us += vu[u];
      }
  }
  const float ns = tk_misc().norm_scale;
  gs *= ns;
  us *= ns;
  const float act = silu_f32(gs) * us;
  const float sc = pow2_scale_for(warp_max(fabsf(act)));
  const float v = act * (1.f / sc);
  const __half h = __float2half_rn(v);
  p.ws.act_hi[s * 32 + lane] = h;
  p.ws.act_lo[s * 32 + lane] = __float2half_rn(v - __half2float(h));
  if (lane == 0) p.ws.act_scale[s] = sc;
  __threadfence();
  __syncwarp();
  if (lane == 0) {
    p.ws.ticket[s] = 0u;
    red_release_add(&p.ws.sync->act_done, 1u);
  }
}

// Writes the warp's segment of block s (ntiles of its tpr tiles), counts the
// tiles on the block's ticket and returns true when they completed the block
// (the caller then owes the block's activation, tk_act).
__device__ __forceinline__ bool tk_flush_gu(float* gu_part, unsigned* ticket, int s, int seg, int ntiles, int tpr,
                                            int lane, float acc[2][4]) {
  const int g = lane >> 2, t = lane & 3;
  if (t == 0) {
    float* part = gu_part + ((int64_t)s * kMaxUnitsPerSlot + seg) * 64;
#pragma unroll
    for (int pr = 0; pr < 2; ++pr)
#pragma unroll
      for (int i = 0; i < 4; ++i) part[pr * 32 + (i >> 1) * 16 + g + (i & 1) * 8] = acc[pr][i];
    __threadfence();
  }
#pragma unroll
  for (int pr = 0; pr < 2; ++pr)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[pr][i] = 0.f;
  __syncwarp();
  unsigned old = 0u;
  if (lane == 0) old = atomicAdd(ticket + s, (unsigned)ntiles);
  old = __shfl_sync(0xffffffffu, old, 0);
  return old + (unsigned)ntiles == (unsigned)tpr;
}

__device__ __forceinline__ void tk_gateup(const TkParams& p, const TkLayer& L, int count) {
  char* sm = tk_smem();
  const TkMisc& M = tk_misc();
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, warp = threadIdx.x >> 5;
  const int warp_global = blockIdx.x * kTkWarps + warp;
  const int tpr = p.H >> 6;
  const int total = count * tpr;
  const int nw = stream_warps(count, tpr, kMaxUnitsPerSlot, (int)gridDim.x * kTkWarps);
  if (count <= 0 || warp_global >= nw) return;
  const int q0 = stream_begin(total, nw, warp_global), q1 = stream_begin(total, nw, warp_global + 1);
  const int* srows = reinterpret_cast<const int*>(sm + kTkRowsOff);
  const uint32_t lb = (uint32_t)lane * 4u;
  const uint32_t xb = smem_u32(sm + kTkXOff) + ((g & 1) ? (uint32_t)p.H * 2u : 0u) + (uint32_t)t * 32u;
  const float* xss = reinterpret_cast<const float*>(sm + kTkXOff + p.H * 4);
  const float ig = M.inv_alpha[0], iu = M.inv_alpha[1];
  // load cursor: the next tile's gate / up bytes and absmax; block bases are
  // read from the descriptor only when the cursor moves to the next block
  int ls = q0 / tpr, lj = q0 - ls * tpr;
  const uint8_t* gb;
  const uint8_t* ub;
  const float* ga;
  const float* ua;
  auto seek = [&]() {
    const int64_t row = srows[ls];
    gb = L.gate + row * L.gstride + (int64_t)lj * 1024 + lane * 16;
    ub = L.up + row * L.gstride + (int64_t)lj * 1024 + lane * 16;
    ga = L.gate_am + row * L.gastride + lj * 32 + g * 4;
    ua = L.up_am + row * L.gastride + lj * 32 + g * 4;
  };
  seek();
  auto load = [&](TkTile& tl) {
    tl.w[0][0] = ldg_stream_u4(gb);
    tl.w[0][1] = ldg_stream_u4(gb + 512);
    tl.w[1][0] = ldg_stream_u4(ub);
    tl.w[1][1] = ldg_stream_u4(ub + 512);
    tl.am[0] = ldg_f4(ga);
    tl.am[1] = ldg_f4(ua);
    gb += 1024;
    ub += 1024;
    ga += 32;
    ua += 32;
    if (++lj == tpr) {
      lj = 0;
      if (++ls < count) seek();
    }
  };
  TkTile buf[kTkDepthGU];
#pragma unroll
  for (int i = 0; i < kTkDepthGU; ++i)
    if (q0 + i < q1) load(buf[i]);
  const int s_first = q0 / tpr;
  int s = s_first, j = q0 - s * tpr, j_seg = j;  // j_seg: the tile this segment started at
  int seg = warp_global - stream_owner(total, nw, s * tpr);
  unsigned long long owed = 0ull;  // bit s - s_first: this warp finalizes block s
  float acc[2][4] = {};
  for (int q = q0; q < q1; q += kTkDepthGU) {
#pragma unroll
    for (int i = 0; i < kTkDepthGU; ++i) {
      if (q + i < q1) {
        const TkTile tl = buf[i];
        if (q + i + kTkDepthGU < q1) load(buf[i]);
        const uint4 x0 = lds_u4(xb + (uint32_t)j * 128u), x1 = lds_u4(xb + (uint32_t)j * 128u + 16u);
        const uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        const float xs = xss[j];
        tk_tile(tl, bx, xs * ig, xs * iu, lb, acc);
        if (++j == tpr || q + i + 1 == q1) {
          // a warp's range spans at most 3 blocks when blocks are longer than 62
          // tiles, and its length is at most 2 tiles otherwise: s - s_first < 64
          if (tk_flush_gu(p.ws.gu_part, p.ws.ticket, s, seg, j - j_seg, tpr, lane, acc))
            owed |= 1ull << ((s - s_first) & 63);
          seg = 0;
          j_seg = j;
          if (j == tpr) {
            j = 0;
            j_seg = 0;
            ++s;
          }
        }
      }
    }
  }
  // the activations of the blocks whose last tiles this warp flushed
  while (owed) {
    const int b = __ffsll((long long)owed) - 1;
    owed &= owed - 1ull;
    tk_act(p, s_first + b, total, nw, tpr);
  }
}

// ---- down: direct-load stream over (64-row group, block) pairs, row-group major -----
struct TkDn {
  uint4 w0, w1;   // the two 32-row tiles: lane (g, t) bytes [4t, 4t+4) of rows g, g+8, 16+g, 24+g
  float4 a0, a1;  // their absmax
};

template <int kTable>
__device__ __forceinline__ void tk_down_mma(uint32_t lb, uint32_t w0, uint32_t w1, const uint4 bf, float d[4]) {
  mma_16816_z(d, lut_get<0x400>(w0, lb, 0, kTable), lut_get<0x400>(w1, lb, 0, kTable),
              lut_get<0x400>(w0, lb, 1, kTable), lut_get<0x400>(w1, lb, 1, kTable), bf.x, bf.y);
  mma_16816(d, lut_get<0x400>(w0, lb, 2, kTable), lut_get<0x400>(w1, lb, 2, kTable),
            lut_get<0x400>(w0, lb, 3, kTable), lut_get<0x400>(w1, lb, 3, kTable), bf.z, bf.w);
}

// The down loop of one layer, with the CTA's wait for every block's
// activation in the middle: each warp first issues the loads of its first
// pairs (weights do not depend on the activations).  next != null: the
// router slices of the next layer are prefetched once the activations are
// staged.  Returns false on abort.
template <int kTable>
__device__ __forceinline__ bool tk_down(const TkParams& p, const TkLayer& L, int count, const TkLayer* next) {
  char* sm = tk_smem();
  TkMisc& M = tk_misc();
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, warp = threadIdx.x >> 5;
  const int warp_global = blockIdx.x * kTkWarps + warp;
  const int RP = p.H >> 6, total = RP * count;
  const int nw = stream_warps(RP, count, kMaxSlotGroups, (int)gridDim.x * kTkWarps);
  const bool active = count > 0 && warp_global < nw;
  const int q0 = active ? stream_begin(total, nw, warp_global) : 0;
  const int q1 = active ? stream_begin(total, nw, warp_global + 1) : 0;
  const int* srows = reinterpret_cast<const int*>(sm + kTkRowsOff);
  const uint8_t* const down = L.down;
  const float* const down_am = L.down_am;
  const int64_t dbs = L.dbs, dabs = L.dabs;
  float* const ypart = p.ws.ypart;
  int lrp = active ? q0 / count : 0, ls = active ? q0 - lrp * count : 0;  // load cursor
  auto load = [&](TkDn& dn) {
    const int64_t row = srows[ls];
    const uint8_t* base = down + row * dbs + (int64_t)lrp * 1024 + lane * 16;
    dn.w0 = ldg_stream_u4(base);
    dn.w1 = ldg_stream_u4(base + 512);
    const float* am = down_am + row * dabs + lrp * 64 + g * 4;
    dn.a0 = ldg_f4(am);
    dn.a1 = ldg_f4(am + 32);
    if (++ls == count) {
      ls = 0;
      ++lrp;
    }
  };
  TkDn buf[kTkDepthDn];
#pragma unroll
  for (int i = 0; i < kTkDepthDn; ++i)
    if (q0 + i < q1) load(buf[i]);
  // every warp of this CTA is past gate/up; wait for all blocks' activations
  __syncthreads();
  if (threadIdx.x == 0) M.act_target += (unsigned)count;
  if (!tk_wait(p, &p.ws.sync->act_done, M.act_target)) return false;
  if (threadIdx.x == 0 && p.ws.sync->stamps != nullptr && M.layer < p.ws.sync->stamp_layers)
    p.ws.sync->stamps[((int64_t)M.layer * gridDim.x + blockIdx.x) * kTkStamps + 6] = tk_now();
  {
    uint4* dst = reinterpret_cast<uint4*>(sm + kTkXOff);
    const int n16 = count * 4;  // 16-byte chunks of one [count][32] fp16 array
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
      const uint4 a = __ldcg(reinterpret_cast<const uint4*>(p.ws.act_hi) + i);
      const uint4 b = __ldcg(reinterpret_cast<const uint4*>(p.ws.act_lo) + i);
      dst[i] = a;
      dst[n16 + i] = b;
    }
    float* sc = reinterpret_cast<float*>(sm + kTkXOff + count * 128);
    for (int i = threadIdx.x; i < count; i += blockDim.x) sc[i] = ldcg_f32(p.ws.act_scale + i);
  }
  __syncthreads();
  if (next != nullptr && warp == 0) {
    tk_prefetch_router(p, *next);
    if (lane == 0) M.pf_out = 1;
  }
  if (!active) return true;
  const uint32_t lb = (uint32_t)lane * 4u;
  const uint32_t ab = smem_u32(sm + kTkXOff) + ((g & 1) ? (uint32_t)count * 64u : 0u) + (uint32_t)t * 16u;
  const float* sc = reinterpret_cast<const float*>(sm + kTkXOff + count * 128);
  const float inv_d = M.inv_alpha[kTable];
  int rp = q0 / count, s = q0 - rp * count;
  int seg = warp_global - stream_owner(total, nw, rp * count);
  float acc[2][4] = {};
  for (int q = q0; q < q1; q += kTkDepthDn) {
#pragma unroll
    for (int i = 0; i < kTkDepthDn; ++i) {
      if (q + i < q1) {
        const TkDn dn = buf[i];
        if (q + i + kTkDepthDn < q1) load(buf[i]);
        const uint4 bf = lds_u4(ab + (uint32_t)s * 64u);
        const float as = sc[s] * inv_d;
        float d[4];
        tk_down_mma<kTable>(lb, dn.w0.x, dn.w0.y, bf, d);
        acc[0][0] = fmaf(d[0] + d[1], dn.a0.x * as, acc[0][0]);
        acc[0][1] = fmaf(d[2] + d[3], dn.a0.y * as, acc[0][1]);
        tk_down_mma<kTable>(lb, dn.w0.z, dn.w0.w, bf, d);
        acc[0][2] = fmaf(d[0] + d[1], dn.a0.z * as, acc[0][2]);
        acc[0][3] = fmaf(d[2] + d[3], dn.a0.w * as, acc[0][3]);
        tk_down_mma<kTable>(lb, dn.w1.x, dn.w1.y, bf, d);
        acc[1][0] = fmaf(d[0] + d[1], dn.a1.x * as, acc[1][0]);
        acc[1][1] = fmaf(d[2] + d[3], dn.a1.y * as, acc[1][1]);
        tk_down_mma<kTable>(lb, dn.w1.z, dn.w1.w, bf, d);
        acc[1][2] = fmaf(d[0] + d[1], dn.a1.z * as, acc[1][2]);
        acc[1][3] = fmaf(d[2] + d[3], dn.a1.w * as, acc[1][3]);
        if (++s == count || q + i + 1 == q1) {
          if (t == 0) {
            float* yp = ypart + (int64_t)seg * p.H + rp * 64;
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
              for (int c = 0; c < 4; ++c) yp[r * 32 + (c >> 1) * 16 + g + (c & 1) * 8] = acc[r][c];
          }
#pragma unroll
          for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
          seg = 0;
          if (s == count) {
            s = 0;
            ++rp;
          }
        }
      }
    }
  }
  return true;
}

// ---- the token kernel ---------------------------------------------------------------
__global__ void __launch_bounds__(kTkThreads, 1) token_kernel(TkParams p) {
  TkMisc& M = tk_misc();
  TkSync* sync = p.ws.sync;
  const int tid = threadIdx.x, cta = blockIdx.x, G = (int)gridDim.x;
  const uint32_t bar = smem_u32(tk_smem() + kTkBarOff);
  const uint32_t xbar = bar + 8u;
  if (tid == 0) {
    M.abort = 0;
    M.count_prev = 0;
    M.act_target = 0u;
    M.bar_phase = 0u;
    M.pf_out = 0;
    M.x_phase = 0u;
    M.x_out = 0;
    M.layer = 0;
    mbar_init(bar, 1);
    mbar_init(xbar, 1);
  }
  mbar_init_fence();
  __syncthreads();
  if (lut_base_addr() != 0x400u) {
    if (tid == 0) tk_fail(p, NSM_ERR_UNSUPPORTED);  // the lookups address the table at 0x400
    __syncthreads();
  }
  const int nA = p.H / kTkCols;
  const uint32_t base = p.ex.world > 1 ? (uint32_t)ld_volatile_i32(reinterpret_cast<const int*>(p.ex.counter)) : 0u;
  const TkLayer* Ls = p.ws.layers;
  if (!M.abort && p.L > 0) {
    tk_build_lut(p, Ls[0]);
    if (tid < 32) {
      tk_prefetch_router(p, Ls[0]);
      if (tid == 0) M.pf_out = 1;
    }
  }
  __syncthreads();
  unsigned long long* stamps = sync->stamps;
  const int stamp_layers = sync->stamp_layers;
  auto stamp = [&](int l, int i) {
    if (stamps != nullptr && threadIdx.x == 0 && l < stamp_layers)
      stamps[((int64_t)l * G + cta) * kTkStamps + i] = tk_now();
  };
  for (int l = 0; l < p.L && !M.abort; ++l) {
    const TkLayer& L = Ls[l];
    if (tid == 0) M.layer = l;
    stamp(l, 0);
    // A: the previous layer's output, residual, norm, x, partial latents
    if (cta < nA) {
      if (l > 0 && !tk_wait(p, &sync->y_done, (unsigned)G * (unsigned)l)) break;
      if (!tk_wait_router(p)) break;
      tk_phase_a(p, L, l, cta * kTkCols, l > 0, M.count_prev, base + (uint32_t)l);
      __syncthreads();
      if (M.abort) break;
      tk_arrive(&sync->a_done);
      stamp(l, 1);
    }
    // B: latent, norm scale, scores (x lands in shared memory meanwhile)
    if (!tk_wait(p, &sync->a_done, (unsigned)nA * (unsigned)(l + 1))) break;
    if (!tk_wait_router(p)) break;
    stamp(l, 2);
    if (tid == 0) tk_issue_x(p, xbar);
    tk_phase_b(p, L);
    tk_arrive(&sync->b_done);
    if (tid == 0) {
      M.bar_phase ^= 1u;
      M.pf_out = 0;
    }
    stamp(l, 3);
    // C: selection
    if (!tk_wait(p, &sync->b_done, (unsigned)G * (unsigned)(l + 1))) break;
    if (!tk_codes_match(L)) tk_build_lut(p, L);
    if (M.abort) break;
    const int count = tk_phase_c(p, L, l);
    if (tid == 0) {
      if (!mbar_wait(xbar, M.x_phase, p.wait_spins)) tk_fail(p, NSM_ERR_TIMEOUT);
      M.x_phase ^= 1u;
      M.x_out = 0;
    }
    __syncthreads();
    if (M.abort) break;
    stamp(l, 4);
    // gate/up, activations, down
    tk_gateup(p, L, count);
    stamp(l, 5);
    const TkLayer* next = l + 1 < p.L ? &Ls[l + 1] : nullptr;
    const bool ok = M.down_table == 0 ? tk_down<0>(p, L, count, next) : tk_down<1>(p, L, count, next);
    __syncthreads();
    if (!ok || M.abort) break;
    tk_arrive(&sync->y_done);
    stamp(l, 7);
    if (tid == 0) M.count_prev = count;
  }
  // the last layer's output
  if (!M.abort && cta < nA && p.L > 0) {
    if (tk_wait(p, &sync->y_done, (unsigned)G * (unsigned)p.L)) {
      const int c0 = cta * kTkCols;
      if (tk_pending_output(p, c0, M.count_prev, base + (uint32_t)p.L) && tid < kTkCols)
        p.residual[c0 + tid] += M.xs[tid];
    }
  }
  __syncthreads();
  // copies still in flight land before the CTA leaves
  if (tid == 0 && M.pf_out) mbar_wait(bar, M.bar_phase);
  if (tid == 0 && M.x_out) mbar_wait(xbar, M.x_phase);
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned old = atomicAdd(&sync->exit_count, 1u);
    if (old == (unsigned)G - 1u) {
      // every other CTA is done with the counters: reset them for the next token
      __threadfence();
      sync->y_done = 0u;
      sync->a_done = 0u;
      sync->b_done = 0u;
      sync->act_done = 0u;
      if (ld_volatile_i32(&sync->err) != 0)
        for (int i = 0; i < kTkMaxK; ++i) p.ws.ticket[i] = 0u;
      else if (p.ex.world > 1)
        *p.ex.counter = base + (uint32_t)p.L;
      __threadfence();
      sync->exit_count = 0u;
    }
  }
}

}  // namespace nsm

using namespace nsm;

// ---- host side -----------------------------------------------------------------------
namespace {

std::mutex g_tk_mu;
int g_tk_setup[64] = {};

int tk_setup(const DeviceInfo& d) {
  std::lock_guard<std::mutex> lk(g_tk_mu);
  if (g_tk_setup[d.device]) return NSM_OK;
  NSM_CHECK_CUDA(cudaFuncSetAttribute(token_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTkSmem));
  int per_sm = 0;
  NSM_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, token_kernel, kTkThreads, kTkSmem));
  if (per_sm < 1) return fail(NSM_ERR_UNSUPPORTED, "the token kernel does not fit on an SM");
  g_tk_setup[d.device] = 1;
  return NSM_OK;
}

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

int tk_shape_ok(int hidden, int intermediate, const DeviceInfo& d) {
  NSM_REQUIRE(hidden > 0 && hidden % kTkCols == 0 && hidden <= kTkMaxH, NSM_ERR_UNSUPPORTED,
              "nsm_decode_token: hidden must be a multiple of 128, at most 16384");
  NSM_REQUIRE(hidden / kTkCols <= d.sm_count, NSM_ERR_UNSUPPORTED, "nsm_decode_token: hidden too large for the grid");
  NSM_REQUIRE(intermediate > 0 && intermediate % 64 == 0, NSM_ERR_UNSUPPORTED,
              "nsm_decode_token: intermediate must be a positive multiple of 64");
  const int NB = intermediate / 32;
  NSM_REQUIRE(NB <= kTkMaxNB && NB <= kTkMaxScoreRows * d.sm_count, NSM_ERR_UNSUPPORTED,
              "nsm_decode_token: at most 4096 blocks");
  return NSM_OK;
}

}  // namespace

extern "C" {

size_t nsm_token_workspace_bytes(int hidden, int intermediate, int num_layers) {
  if (hidden <= 0 || intermediate <= 0 || num_layers <= 0) return 0;
  return tk_ws_layout(nullptr, hidden, intermediate / 32, num_layers).bytes;
}

int nsm_token_set_layers(void* ws, size_t ws_bytes, int32_t hidden, int32_t intermediate,
                         const nsm_token_layer* layers, int32_t num_layers, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  st = tk_shape_ok(hidden, intermediate, dev);
  if (st) return st;
  NSM_REQUIRE(layers != nullptr && num_layers > 0, NSM_ERR_INVALID_ARG, "nsm_token_set_layers: no layers");
  const int NB = intermediate / 32;
  const TkWs w = tk_ws_layout(ws, hidden, NB, num_layers);
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= w.bytes, NSM_ERR_WORKSPACE,
              "nsm_token_set_layers: workspace smaller than nsm_token_workspace_bytes");
  std::vector<TkLayer> dl((size_t)num_layers);
  for (int i = 0; i < num_layers; ++i) {
    const nsm_token_layer& in = layers[i];
    const nsm_router_weights& r = in.router;
    const nsm_mlp_weights& m = in.mlp;
    NSM_REQUIRE(r.enc_w && r.score_w && aligned16(r.enc_w) && aligned16(r.score_w), NSM_ERR_INVALID_ARG,
                "nsm_token_set_layers: router weights missing or not 16-byte aligned");
    NSM_REQUIRE(r.weight_dtype == NSM_BF16 || r.weight_dtype == NSM_F16, NSM_ERR_UNSUPPORTED,
                "nsm_token_set_layers: router weights must be bf16 or fp16");
    NSM_REQUIRE(r.rank == kTkRank, NSM_ERR_UNSUPPORTED, "nsm_token_set_layers: router rank must be 64");
    NSM_REQUIRE(r.num_blocks == NB, NSM_ERR_INVALID_ARG, "nsm_token_set_layers: router num_blocks != intermediate/32");
    NSM_REQUIRE(r.top_k > 0 && std::min(r.top_k, NB) <= kTkMaxK, NSM_ERR_UNSUPPORTED,
                "nsm_token_set_layers: top_k must be in [1, 256]");
    NSM_REQUIRE((m.layout & NSM_LAYOUT_GATEUP_TILED) && (m.layout & NSM_LAYOUT_DOWN_TILED), NSM_ERR_UNSUPPORTED,
                "nsm_token_set_layers: the pools must use the tiled layouts");
    NSM_REQUIRE(!m.gate_bias && !m.up_bias && !m.down_bias, NSM_ERR_UNSUPPORTED,
                "nsm_token_set_layers: biases are not supported on this path");
    NSM_REQUIRE(m.gate_packed && m.gate_absmax && m.up_packed && m.up_absmax && m.down_packed && m.down_absmax &&
                    m.gate_code && m.up_code && m.down_code && m.pool_rows > 0,
                NSM_ERR_INVALID_ARG, "nsm_token_set_layers: an MLP pointer is NULL or pool_rows is 0");
    const int64_t gs = m.gateup_block_stride ? m.gateup_block_stride : (int64_t)16 * hidden;
    const int64_t gas = m.gateup_absmax_block_stride ? m.gateup_absmax_block_stride : (int64_t)hidden / 2;
    const int64_t dbs = m.down_block_stride ? m.down_block_stride : (int64_t)16 * hidden;
    const int64_t das = m.down_absmax_block_stride ? m.down_absmax_block_stride : (int64_t)hidden;
    NSM_REQUIRE(aligned16(m.gate_packed) && aligned16(m.up_packed) && aligned16(m.gate_absmax) &&
                    aligned16(m.up_absmax) && aligned16(m.down_packed) && aligned16(m.down_absmax) && gs % 16 == 0 &&
                    (gas * 4) % 16 == 0 && dbs % 16 == 0 && (das * 4) % 16 == 0,
                NSM_ERR_INVALID_ARG, "nsm_token_set_layers: pools and strides must be 16-byte aligned");
    NSM_REQUIRE(in.norm_weight == nullptr ||
                    ((in.norm_weight_dtype == NSM_F32 || in.norm_weight_dtype == NSM_F16 ||
                      in.norm_weight_dtype == NSM_BF16) &&
                     aligned16(in.norm_weight)),
                NSM_ERR_INVALID_ARG, "nsm_token_set_layers: bad norm weight");
    TkLayer& o = dl[(size_t)i];
    o = TkLayer{};
    o.enc_w = r.enc_w;
    o.enc_b = r.enc_b;
    o.score_w = r.score_w;
    o.score_b = r.score_b;
    o.dbn = r.down_block_norm;
    o.norm_w = in.norm_weight;
    o.gate = m.gate_packed;
    o.gate_am = m.gate_absmax;
    o.up = m.up_packed;
    o.up_am = m.up_absmax;
    o.down = m.down_packed;
    o.down_am = m.down_absmax;
    o.gate_code = m.gate_code;
    o.up_code = m.up_code;
    o.down_code = m.down_code;
    o.slot_of_block = in.map.slot_of_block;
    o.gstride = gs;
    o.gastride = gas;
    o.dbs = dbs;
    o.dabs = das;
    o.wdtype = r.weight_dtype;
    o.norm_dtype = in.norm_weight_dtype;
    o.top_k = r.top_k;
    o.basis_top_k = r.basis_top_k;
    o.legacy = r.legacy_abs_latent;
    o.pool_rows = m.pool_rows;
    o.block_begin = in.map.slot_of_block ? 0 : in.map.block_begin;
    o.block_end = in.map.slot_of_block ? NB : in.map.block_end;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  NSM_CHECK_CUDA(cudaMemcpyAsync(w.layers, dl.data(), dl.size() * sizeof(TkLayer), cudaMemcpyHostToDevice, s));
  NSM_CHECK_CUDA(cudaStreamSynchronize(s));
  return NSM_OK;
}

int nsm_token_profile(void* ws, size_t ws_bytes, int32_t hidden, int32_t intermediate, int32_t num_layers,
                      unsigned long long* stamps, int32_t stamp_layers, nsm_stream_t stream) {
  NSM_REQUIRE(hidden > 0 && intermediate > 0 && num_layers > 0, NSM_ERR_INVALID_ARG, "nsm_token_profile: bad shape");
  const TkWs w = tk_ws_layout(ws, hidden, intermediate / 32, num_layers);
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= w.bytes, NSM_ERR_WORKSPACE, "nsm_token_profile: workspace missing, not 256-byte aligned or too small");
  NSM_REQUIRE(stamps == nullptr || stamp_layers > 0, NSM_ERR_INVALID_ARG, "nsm_token_profile: stamp_layers <= 0");
  unsigned long long* sp = stamps;
  int n = stamps ? stamp_layers : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  NSM_CHECK_CUDA(cudaMemcpyAsync(&w.sync->stamps, &sp, sizeof(sp), cudaMemcpyHostToDevice, s));
  NSM_CHECK_CUDA(cudaMemcpyAsync(&w.sync->stamp_layers, &n, sizeof(n), cudaMemcpyHostToDevice, s));
  NSM_CHECK_CUDA(cudaStreamSynchronize(s));
  return NSM_OK;
}

int nsm_decode_token(float* residual, int32_t hidden, int32_t intermediate, int32_t num_layers, float eps,
                     const nsm_exchange* ex, int32_t* trace_blocks, int32_t trace_k, int32_t* trace_counts,
                     float* trace_residual, void* ws, size_t ws_bytes, nsm_stream_t stream) {
  DeviceInfo dev;
  int st = current_device(&dev);
  if (st) return st;
  st = tk_shape_ok(hidden, intermediate, dev);
  if (st) return st;
  NSM_REQUIRE(residual != nullptr, NSM_ERR_INVALID_ARG, "nsm_decode_token: residual is NULL");
  NSM_REQUIRE(num_layers > 0, NSM_ERR_INVALID_ARG, "nsm_decode_token: num_layers must be > 0");
  NSM_REQUIRE(trace_blocks == nullptr || trace_k > 0, NSM_ERR_INVALID_ARG, "nsm_decode_token: trace_k must be > 0");
  const int NB = intermediate / 32;
  const TkWs w = tk_ws_layout(ws, hidden, NB, num_layers);
  NSM_REQUIRE(ws != nullptr && ((uintptr_t)ws & 255) == 0 && ws_bytes >= w.bytes, NSM_ERR_WORKSPACE,
              "nsm_decode_token: workspace smaller than nsm_token_workspace_bytes");
  st = tk_setup(dev);
  if (st) return st;
  TkParams p{};
  p.ws = w;
  p.residual = residual;
  p.H = hidden;
  p.NB = NB;
  p.L = num_layers;
  p.eps = eps;
  if (ex != nullptr) {
    const ExchangeDev* e = exchange_dev(ex);
    NSM_REQUIRE(e->hidden == hidden && e->data[0] != nullptr, NSM_ERR_INVALID_ARG,
                "nsm_decode_token: exchange not connected or built for another hidden size");
    p.ex = *e;
  } else {
    p.ex.world = 1;
  }
  p.wait_spins = copy_wait_spins();
  p.trace_blocks = trace_blocks;
  p.trace_counts = trace_counts;
  p.trace_residual = trace_residual;
  p.trace_k = trace_k;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)dev.sm_count);
  cfg.blockDim = dim3(kTkThreads);
  cfg.dynamicSmemBytes = kTkSmem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  NSM_CHECK_CUDA(cudaLaunchKernelEx(&cfg, token_kernel, p));
  return NSM_OK;
}

}  // extern "C"
