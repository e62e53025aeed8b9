// nsm_aux.cu -- layout repack, the reference's generic 4-bit linear API
// semantics, and the device side of the VRAM hot-block cache.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "nsm_common.cuh"
#include "nsm_internal.h"

namespace nsm {

constexpr int kStageMaxJobs = 256;  // records per gather launch (the pointers travel in the parameters)
constexpr int kStageThreads = 256;
constexpr int kStageVec = 8;        // 16-byte loads in flight per thread
struct StageParams {
  const uint4* src[kStageMaxJobs];  // device view of the host record
  uint4* dst[kStageMaxJobs];        // pool row
  int64_t vecs;                     // 16-byte vectors per record
  int n;
};
const char* stage_device_view(const void* host);
__global__ void cache_stage_gather_kernel(const __grid_constant__ StageParams p);

// ---------------------------------------------------------------------------
// down weight [H][I/2] (+ absmax [H][I/64]) -> block-major [n][H][16] + [n][H]
// ---------------------------------------------------------------------------
__global__ void repack_down_kernel(const uint8_t* __restrict__ src, const float* __restrict__ src_am, int H, int I,
                                   const int32_t* __restrict__ blocks, int n, uint8_t* __restrict__ dst,
                                   float* __restrict__ dst_am) {
  const int64_t total = (int64_t)n * H;
  const int64_t bpr = I / 2, apr = I / 64;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int slot = (int)(i / H), h = (int)(i - (int64_t)slot * H);
    const int b = blocks ? blocks[slot] : slot;
    const uint4 v = *reinterpret_cast<const uint4*>(src + (int64_t)h * bpr + (int64_t)b * 16);
    *reinterpret_cast<uint4*>(dst + ((int64_t)slot * H + h) * 16) = v;
    dst_am[(int64_t)slot * H + h] = src_am[(int64_t)h * apr + (b >> 1)];
  }
}

// ---------------------------------------------------------------------------
// bitsandbytes row-major -> tiled pool rows (layout documented in nsm.h)
// ---------------------------------------------------------------------------
struct RepackParams {
  const uint8_t* src_pk[3];  // gate, up, down
  const float* src_am[3];
  uint8_t* dst_pk[3];
  float* dst_am[3];
  int64_t dst_pk_stride[3];  // bytes between destination rows
  int64_t dst_am_stride[3];  // floats between destination rows
  int H, I;
  const int32_t* blocks;
  const int32_t* dst_rows;
  int n;
};

// blockIdx.y: 0/1 gate/up packed, 2/3 gate/up absmax, 4 down packed, 5 down absmax
__global__ void repack_tiled_kernel(RepackParams p) {
  const int part = blockIdx.y;
  const int H = p.H;
  const int proj = part < 2 ? part : (part < 4 ? part - 2 : 2);
  const bool is_am = part == 2 || part == 3 || part == 5;
  if (is_am ? p.src_am[proj] == nullptr : p.src_pk[proj] == nullptr) return;
  int64_t per_block;  // outputs per block
  if (part < 2) per_block = H;            // 16-byte chunks
  else if (part < 4) per_block = H / 8;   // float4s
  else if (part == 4) per_block = H;      // 16-byte chunks
  else per_block = H / 4;                 // float4s
  const int64_t total = per_block * p.n;
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(q / per_block);
    const int64_t c = q - (int64_t)i * per_block;
    const int b = p.blocks ? p.blocks[i] : i;
    const int d = p.dst_rows ? p.dst_rows[i] : i;
    if (part < 2) {
      const int j = (int)(c >> 6), rem = (int)(c & 63), rg = rem >> 5, lane = rem & 31;
      const int g = lane >> 2, t = lane & 3;
      const uint8_t* src = p.src_pk[proj] + (int64_t)b * 16 * H;
      const int r0 = rg * 16 + g;
      const uint2 a = *reinterpret_cast<const uint2*>(src + (int64_t)r0 * (H / 2) + j * 32 + t * 8);
      const uint2 e = *reinterpret_cast<const uint2*>(src + (int64_t)(r0 + 8) * (H / 2) + j * 32 + t * 8);
      *reinterpret_cast<uint4*>(p.dst_pk[proj] + d * p.dst_pk_stride[proj] + (int64_t)c * 16) =
          make_uint4(a.x, a.y, e.x, e.y);
    } else if (part < 4) {
      const int j = (int)(c >> 3), g = (int)(c & 7);
      const float* src = p.src_am[proj] + (int64_t)b * (H / 2);
      const int apr = H / 64;
      const float4 v = make_float4(src[(int64_t)g * apr + j], src[(int64_t)(g + 8) * apr + j],
                                   src[(int64_t)(g + 16) * apr + j], src[(int64_t)(g + 24) * apr + j]);
      *reinterpret_cast<float4*>(p.dst_am[proj] + d * p.dst_am_stride[proj] + c * 4) = v;
    } else if (part == 4) {
      const int rt = (int)(c >> 5), lane = (int)(c & 31), g = lane >> 2, t = lane & 3;
      const uint8_t* src = p.src_pk[2] + (int64_t)b * 16 + t * 4;
      const int64_t bpr = p.I / 2;
      const int r0 = rt * 32 + g;
      const uint4 v = make_uint4(*reinterpret_cast<const uint32_t*>(src + (int64_t)r0 * bpr),
                                 *reinterpret_cast<const uint32_t*>(src + (int64_t)(r0 + 8) * bpr),
                                 *reinterpret_cast<const uint32_t*>(src + (int64_t)(r0 + 16) * bpr),
                                 *reinterpret_cast<const uint32_t*>(src + (int64_t)(r0 + 24) * bpr));
      *reinterpret_cast<uint4*>(p.dst_pk[2] + d * p.dst_pk_stride[2] + (int64_t)c * 16) = v;
    } else {
      const int rt = (int)(c >> 3), g = (int)(c & 7);
      const int64_t apr = p.I / 64;
      const float* src = p.src_am[2] + (b >> 1);
      const int r0 = rt * 32 + g;
      const float4 v = make_float4(src[(int64_t)r0 * apr], src[(int64_t)(r0 + 8) * apr], src[(int64_t)(r0 + 16) * apr],
                                   src[(int64_t)(r0 + 24) * apr]);
      *reinterpret_cast<float4*>(p.dst_am[2] + d * p.dst_am_stride[2] + c * 4) = v;
    }
  }
}

// ---------------------------------------------------------------------------
// triton_sparse_input_linear_4bit semantics (NF4 of weight.t(): element index
// e = in_idx * out_features + out_idx).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float nf4_elem(const uint8_t* packed, const float* absmax, const float* code, int64_t e,
                                          int qbs) {
  const uint8_t byte = packed[e >> 1];
  const int nib = (e & 1) ? (byte & 0x0f) : (byte >> 4);
  return code[nib] * absmax[e / qbs];
}

__global__ void input_linear_4bit_kernel(const void* x, int dt, int rows, const int32_t* idx, int k,
                                         const uint8_t* packed, const float* absmax, const float* code, int out_f,
                                         int in_f, int qbs, const void* bias, int bs, void* out) {
  __shared__ float scode[16];
  if (threadIdx.x < 16) scode[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  const int r = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= out_f) return;
  float acc = bias ? load_as_f32(bias, dt, n) : 0.f;
  for (int s = 0; s < k; ++s) {
    const int blk = idx[(int64_t)r * k + s];
    if (blk < 0) continue;
    for (int i = 0; i < bs; ++i) {
      const int col = blk * bs + i;
      if (col >= in_f) break;
      const int64_t e = (int64_t)col * out_f + n;
      acc = fmaf(nf4_elem(packed, absmax, scode, e, qbs), load_as_f32(x, dt, (int64_t)r * in_f + col), acc);
    }
  }
  store_from_f32(out, dt, (int64_t)r * out_f + n, acc);
}

// triton_sparse_output_linear_4bit semantics: e = k*bs + blk*bs + o.
__global__ void output_linear_4bit_kernel(const void* x, int dt, int rows, const int32_t* idx, int k,
                                          const void* mask, int width, const uint8_t* packed, const float* absmax,
                                          const float* code, int din, int qbs, const void* bias, int bs, void* out) {
  __shared__ float scode[16];
  if (threadIdx.x < 16) scode[threadIdx.x] = code[threadIdx.x];
  __syncthreads();
  const int r = blockIdx.y / k, s = blockIdx.y - (blockIdx.y / k) * k;
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= bs) return;
  const int blk = idx[(int64_t)r * k + s];
  if (blk < 0) return;
  const int col = blk * bs + o;
  if (col >= width) return;
  float acc = bias ? load_as_f32(bias, dt, col) : 0.f;
  for (int kk = 0; kk < din; ++kk) {
    const int64_t e = (int64_t)kk * bs + col;
    acc = fmaf(nf4_elem(packed, absmax, scode, e, qbs), load_as_f32(x, dt, (int64_t)r * din + kk), acc);
  }
  const float m = mask ? load_as_f32(mask, dt, (int64_t)r * width + col) : 1.f;
  store_from_f32(out, dt, (int64_t)r * width + col, acc * m);
}

// ---------------------------------------------------------------------------
// hot-block cache
// ---------------------------------------------------------------------------
__global__ void cache_split_kernel(const int32_t* idx, int k, const int32_t* slot_of_block, int nb, int32_t* hit_rows,
                                   int32_t* miss_pos, int32_t* counts) {
  __shared__ int wh[32], wm[32];
  __shared__ int base_h, base_m;
  if (threadIdx.x == 0) base_h = base_m = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int j0 = 0; j0 < k; j0 += blockDim.x) {
    const int j = j0 + threadIdx.x;
    int row = -1;
    bool valid = false;
    if (j < k) {
      const int b = idx[j];
      valid = b >= 0 && b < nb;
      row = valid ? slot_of_block[b] : -1;
    }
    const bool hit = valid && row >= 0;
    const bool miss = valid && row < 0;
    const unsigned bh = __ballot_sync(0xffffffffu, hit), bm = __ballot_sync(0xffffffffu, miss);
    if (lane == 0) {
      wh[warp] = __popc(bh);
      wm[warp] = __popc(bm);
    }
    __syncthreads();
    int oh = 0, om = 0;
    for (int w = 0; w < warp; ++w) {
      oh += wh[w];
      om += wm[w];
    }
    const unsigned lt = (1u << lane) - 1u;
    if (hit) hit_rows[base_h + oh + __popc(bh & lt)] = row;
    if (miss) miss_pos[base_m + om + __popc(bm & lt)] = j;
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 0; w < nw; ++w) {
        base_h += wh[w];
        base_m += wm[w];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    counts[0] = base_h;
    counts[1] = base_m;
  }
}

__device__ __forceinline__ void copy_bytes(uint8_t* dst, const uint8_t* src, int64_t n, int tid, int nthr) {
  const int64_t n16 = n / 16;
  for (int64_t i = tid; i < n16; i += nthr)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (int64_t i = n16 * 16 + tid; i < n; i += nthr) dst[i] = src[i];
}

struct PromoteParams {
  uint8_t* gate;
  float* gate_am;
  uint8_t* up;
  float* up_am;
  uint8_t* down;
  float* down_am;
  int64_t gstride, gastride, dbs, dabs;
  int H;
  const int32_t* src;
  const int32_t* dst;
};

__global__ void cache_promote_copy_kernel(PromoteParams p) {
  const int i = blockIdx.y;
  const int s = p.src[i], d = p.dst[i];
  const int nthr = gridDim.x * blockDim.x, tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t gb = (int64_t)16 * p.H;          // 32 rows * H/2 bytes
  const int64_t gab = (int64_t)(p.H / 2) * 4;    // 32 rows * H/64 floats
  copy_bytes(p.gate + d * p.gstride, p.gate + s * p.gstride, gb, tid, nthr);
  copy_bytes(p.up + d * p.gstride, p.up + s * p.gstride, gb, tid, nthr);
  copy_bytes(reinterpret_cast<uint8_t*>(p.gate_am + d * p.gastride),
             reinterpret_cast<const uint8_t*>(p.gate_am + s * p.gastride), gab, tid, nthr);
  copy_bytes(reinterpret_cast<uint8_t*>(p.up_am + d * p.gastride),
             reinterpret_cast<const uint8_t*>(p.up_am + s * p.gastride), gab, tid, nthr);
  copy_bytes(p.down + d * p.dbs, p.down + s * p.dbs, (int64_t)16 * p.H, tid, nthr);
  copy_bytes(reinterpret_cast<uint8_t*>(p.down_am + d * p.dabs),
             reinterpret_cast<const uint8_t*>(p.down_am + s * p.dabs), (int64_t)4 * p.H, tid, nthr);
}

__global__ void cache_table_update_kernel(const int32_t* block_ids, const int32_t* evicted, const int32_t* dst, int n,
                                          int32_t* slot_of_block) {
  // evictions first, then installs (single thread keeps the order exact)
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  for (int i = 0; i < n; ++i)
    if (evicted && evicted[i] >= 0) slot_of_block[evicted[i]] = -1;
  for (int i = 0; i < n; ++i) slot_of_block[block_ids[i]] = dst[i];
}

static int dtype_ok(int d) { return d == NSM_F32 || d == NSM_F16 || d == NSM_BF16; }

// ---------------------------------------------------------------------------
// hot-block cache: miss records gathered from pinned host memory
// ---------------------------------------------------------------------------
// The device view of a pinned, mapped host allocation (nullptr for anything
// else: pageable memory must go through the copy engine).
const char* stage_device_view(const void* host) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, host) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type != cudaMemoryTypeHost || a.devicePointer == nullptr) return nullptr;
  return reinterpret_cast<const char*>(a.devicePointer);
}

// Copies whole records: the grid walks (record, 64 KB chunk) items; each
// thread keeps kStageVec 16-byte loads from host memory in flight (a few MB
// over the grid, enough to fill the host link).  No shared memory and few
// registers, so its CTAs fit beside the decode kernels' on the same SMs.
__global__ void __launch_bounds__(kStageThreads) cache_stage_gather_kernel(const __grid_constant__ StageParams p) {
  constexpr int64_t kChunk = (int64_t)kStageThreads * kStageVec * 4;  // 16-byte vectors per item
  const int64_t chunks = (p.vecs + kChunk - 1) / kChunk;
  for (int64_t item = blockIdx.x; item < (int64_t)p.n * chunks; item += gridDim.x) {
    const int j = (int)(item / chunks);
    const int64_t c0 = (item - (int64_t)j * chunks) * kChunk;
    const uint4* src = p.src[j];
    uint4* dst = p.dst[j];
    for (int64_t v0 = c0; v0 < c0 + kChunk && v0 < p.vecs; v0 += (int64_t)kStageThreads * kStageVec) {
      uint4 r[kStageVec];
#pragma unroll
      for (int u = 0; u < kStageVec; ++u) {
        const int64_t v = v0 + (int64_t)u * kStageThreads + threadIdx.x;
        if (v < p.vecs) r[u] = src[v];
      }
#pragma unroll
      for (int u = 0; u < kStageVec; ++u) {
        const int64_t v = v0 + (int64_t)u * kStageThreads + threadIdx.x;
        if (v < p.vecs) dst[v] = r[u];
      }
    }
  }
}

}  // namespace nsm

using namespace nsm;

extern "C" {

int nsm_repack_down_block_major(const uint8_t* down_packed, const float* down_absmax, int32_t hidden,
                                int32_t intermediate, const int32_t* blocks, int32_t n, uint8_t* out_packed,
                                float* out_absmax, nsm_stream_t stream) {
  NSM_REQUIRE(down_packed && down_absmax && out_packed && out_absmax, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(hidden > 0 && intermediate > 0 && intermediate % 64 == 0, NSM_ERR_UNSUPPORTED,
              "intermediate must be a positive multiple of 64");
  NSM_REQUIRE(((uintptr_t)down_packed & 15) == 0 && ((uintptr_t)out_packed & 15) == 0, NSM_ERR_INVALID_ARG,
              "packed pointers must be 16-byte aligned");
  const int nb = intermediate / 32;
  const int cnt = blocks ? n : nb;
  NSM_REQUIRE(cnt > 0, NSM_ERR_INVALID_ARG, "nothing to repack");
  const int64_t total = (int64_t)cnt * hidden;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  repack_down_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(down_packed, down_absmax, hidden,
                                                                                intermediate, blocks, cnt,
                                                                                out_packed, out_absmax);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

int nsm_repack_tiled(const uint8_t* gate_packed, const float* gate_absmax, const uint8_t* up_packed,
                     const float* up_absmax, const uint8_t* down_packed, const float* down_absmax, int32_t hidden,
                     int32_t intermediate, const int32_t* blocks, const int32_t* dst_rows, int32_t n,
                     const nsm_mlp_weights* dst, nsm_stream_t stream) {
  NSM_REQUIRE(dst != nullptr, NSM_ERR_INVALID_ARG, "destination descriptor is NULL");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && intermediate > 0 && intermediate % 64 == 0, NSM_ERR_UNSUPPORTED,
              "hidden and intermediate must be positive multiples of 64");
  const int nb = intermediate / 32;
  const int cnt = blocks ? n : (n > 0 ? n : nb);
  NSM_REQUIRE(cnt > 0, NSM_ERR_INVALID_ARG, "nothing to repack");
  RepackParams p{};
  p.src_pk[0] = gate_packed;
  p.src_pk[1] = up_packed;
  p.src_pk[2] = down_packed;
  p.src_am[0] = gate_absmax;
  p.src_am[1] = up_absmax;
  p.src_am[2] = down_absmax;
  p.dst_pk[0] = const_cast<uint8_t*>(dst->gate_packed);
  p.dst_pk[1] = const_cast<uint8_t*>(dst->up_packed);
  p.dst_pk[2] = const_cast<uint8_t*>(dst->down_packed);
  p.dst_am[0] = const_cast<float*>(dst->gate_absmax);
  p.dst_am[1] = const_cast<float*>(dst->up_absmax);
  p.dst_am[2] = const_cast<float*>(dst->down_absmax);
  const int64_t gs = dst->gateup_block_stride ? dst->gateup_block_stride : (int64_t)16 * hidden;
  const int64_t gas = dst->gateup_absmax_block_stride ? dst->gateup_absmax_block_stride : (int64_t)hidden / 2;
  const int64_t ds = dst->down_block_stride ? dst->down_block_stride : (int64_t)16 * hidden;
  const int64_t das = dst->down_absmax_block_stride ? dst->down_absmax_block_stride : (int64_t)hidden;
  p.dst_pk_stride[0] = p.dst_pk_stride[1] = gs;
  p.dst_am_stride[0] = p.dst_am_stride[1] = gas;
  p.dst_pk_stride[2] = ds;
  p.dst_am_stride[2] = das;
  for (int q = 0; q < 3; ++q) {
    if (p.src_pk[q]) {
      NSM_REQUIRE(p.dst_pk[q] != nullptr, NSM_ERR_INVALID_ARG, "destination packed pointer is NULL");
      NSM_REQUIRE(((uintptr_t)p.dst_pk[q] & 15) == 0 && (p.dst_pk_stride[q] & 15) == 0, NSM_ERR_INVALID_ARG,
                  "destination packed rows must be 16-byte aligned");
      NSM_REQUIRE(((uintptr_t)p.src_pk[q] & (q < 2 ? 7 : 3)) == 0, NSM_ERR_INVALID_ARG, "misaligned source");
    }
    if (p.src_am[q]) {
      NSM_REQUIRE(p.dst_am[q] != nullptr, NSM_ERR_INVALID_ARG, "destination absmax pointer is NULL");
      NSM_REQUIRE(((uintptr_t)p.dst_am[q] & 15) == 0 && (p.dst_am_stride[q] & 3) == 0, NSM_ERR_INVALID_ARG,
                  "destination absmax rows must be 16-byte aligned");
    }
  }
  p.H = hidden;
  p.I = intermediate;
  p.blocks = blocks;
  p.dst_rows = dst_rows;
  p.n = cnt;
  const int64_t work = (int64_t)cnt * hidden;
  const int gx = (int)std::min<int64_t>((work + 255) / 256, 148 * 32);
  repack_tiled_kernel<<<dim3(gx, 6), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

int nsm_sparse_input_linear_4bit(const void* x, int32_t act_dtype, int32_t rows, const int32_t* active_idx,
                                 int32_t top_k, const uint8_t* packed, const float* absmax, const float* code,
                                 int32_t out_features, int32_t in_features, int32_t quant_block_size,
                                 const void* bias, int32_t block_size, void* out, nsm_stream_t stream) {
  NSM_REQUIRE(dtype_ok(act_dtype), NSM_ERR_INVALID_ARG, "bad activation dtype");
  NSM_REQUIRE(block_size > 0, NSM_ERR_INVALID_ARG, "block_size must be > 0 for triton_sparse_input_linear_4bit");
  NSM_REQUIRE(in_features % block_size == 0, NSM_ERR_INVALID_ARG, "in_features must be divisible by block_size");
  NSM_REQUIRE(quant_block_size > 0, NSM_ERR_INVALID_ARG, "quant_block_size must be > 0");
  NSM_REQUIRE(out != nullptr, NSM_ERR_INVALID_ARG, "out is NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows <= 0 || out_features <= 0) return NSM_OK;
  NSM_REQUIRE(x && packed && absmax && code, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(top_k == 0 || active_idx != nullptr, NSM_ERR_INVALID_ARG, "active_idx is NULL");
  dim3 grid((out_features + 255) / 256, rows);
  input_linear_4bit_kernel<<<grid, 256, 0, s>>>(x, act_dtype, rows, active_idx, top_k, packed, absmax, code,
                                                 out_features, in_features, quant_block_size, bias, block_size, out);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

int nsm_sparse_output_linear_4bit(const void* x, int32_t act_dtype, int32_t rows, const int32_t* active_idx,
                                  int32_t top_k, const void* flat_mask, int32_t width, const uint8_t* packed,
                                  const float* absmax, const float* code, int32_t input_dim,
                                  int32_t quant_block_size, const void* bias, int32_t block_size, void* out,
                                  nsm_stream_t stream) {
  NSM_REQUIRE(dtype_ok(act_dtype), NSM_ERR_INVALID_ARG, "bad activation dtype");
  NSM_REQUIRE(block_size > 0, NSM_ERR_INVALID_ARG, "block_size must be > 0 for triton_sparse_output_linear_4bit");
  NSM_REQUIRE(input_dim % block_size == 0, NSM_ERR_INVALID_ARG, "input_dim must be divisible by block_size");
  NSM_REQUIRE(quant_block_size > 0, NSM_ERR_INVALID_ARG, "quant_block_size must be > 0");
  NSM_REQUIRE(out != nullptr && width >= 0, NSM_ERR_INVALID_ARG, "out is NULL");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int es = act_dtype == NSM_F32 ? 4 : 2;
  if (rows <= 0 || width == 0) return NSM_OK;
  NSM_CHECK_CUDA(cudaMemsetAsync(out, 0, (size_t)rows * width * es, s));
  if (top_k <= 0) return NSM_OK;
  NSM_REQUIRE(x && packed && absmax && code && active_idx, NSM_ERR_INVALID_ARG, "NULL pointer");
  dim3 grid((block_size + 127) / 128, rows * top_k);
  output_linear_4bit_kernel<<<grid, 128, 0, s>>>(x, act_dtype, rows, active_idx, top_k, flat_mask, width, packed,
                                                  absmax, code, input_dim, quant_block_size, bias, block_size, out);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

int nsm_cache_split(const int32_t* idx, int32_t k, const int32_t* slot_of_block, int32_t num_blocks, int32_t* hit_rows,
                    int32_t* miss_pos, int32_t* counts, nsm_stream_t stream) {
  NSM_REQUIRE(idx && slot_of_block && hit_rows && miss_pos && counts, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(k > 0 && num_blocks > 0, NSM_ERR_INVALID_ARG, "k and num_blocks must be > 0");
  cache_split_kernel<<<1, 512, 0, reinterpret_cast<cudaStream_t>(stream)>>>(idx, k, slot_of_block, num_blocks,
                                                                            hit_rows, miss_pos, counts);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

int nsm_cache_stage(const void* host_base, int32_t host_records, const int32_t* blocks, int32_t n,
                    size_t record_bytes, void* pool_base, const int32_t* dst_rows, int32_t pool_rows,
                    nsm_stream_t stream) {
  if (n <= 0) return NSM_OK;
  NSM_REQUIRE(host_base && blocks && pool_base && dst_rows, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(record_bytes > 0, NSM_ERR_INVALID_ARG, "record_bytes must be > 0");
  for (int i = 0; i < n; ++i) {
    NSM_REQUIRE(blocks[i] >= 0 && blocks[i] < host_records, NSM_ERR_INVALID_ARG,
                "block id outside the host store");
    NSM_REQUIRE(dst_rows[i] >= 0 && dst_rows[i] < pool_rows, NSM_ERR_INVALID_ARG, "destination row out of range");
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* dst = reinterpret_cast<char*>(pool_base);
  // pinned host memory that the device can address: one gather kernel reads
  // every record over the host link; anything else goes through the copy engine
  const char* dsrc = stage_device_view(host_base);
  if (dsrc != nullptr && record_bytes % 16 == 0 && ((uintptr_t)dsrc | (uintptr_t)dst) % 16 == 0) {
    DeviceInfo dev;
    const int st = current_device(&dev);
    if (st) return st;
    for (int i0 = 0; i0 < n; i0 += kStageMaxJobs) {
      StageParams sp{};
      sp.n = std::min(n - i0, kStageMaxJobs);
      sp.vecs = (int64_t)(record_bytes / 16);
      for (int i = 0; i < sp.n; ++i) {
        sp.src[i] = reinterpret_cast<const uint4*>(dsrc + (size_t)blocks[i0 + i] * record_bytes);
        sp.dst[i] = reinterpret_cast<uint4*>(dst + (size_t)dst_rows[i0 + i] * record_bytes);
      }
      cache_stage_gather_kernel<<<std::max(1, dev.sm_count / 2), kStageThreads, 0, s>>>(sp);
      NSM_CHECK_CUDA(cudaGetLastError());
    }
    return NSM_OK;
  }
  const char* src = reinterpret_cast<const char*>(host_base);
  for (int i = 0; i < n; ++i)
    NSM_CHECK_CUDA(cudaMemcpyAsync(dst + (size_t)dst_rows[i] * record_bytes, src + (size_t)blocks[i] * record_bytes,
                                   record_bytes, cudaMemcpyHostToDevice, s));
  return NSM_OK;
}

int nsm_cache_promote(const nsm_mlp_weights* w, int32_t hidden, const int32_t* src_rows, const int32_t* dst_rows,
                      const int32_t* block_ids, const int32_t* evicted_ids, int32_t n, int32_t* slot_of_block,
                      nsm_stream_t stream) {
  NSM_REQUIRE(w != nullptr, NSM_ERR_INVALID_ARG, "weights descriptor is NULL");
  NSM_REQUIRE(src_rows && dst_rows && block_ids && slot_of_block, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0, NSM_ERR_UNSUPPORTED, "hidden must be a positive multiple of 64");
  const bool down_tiled = (w->layout & NSM_LAYOUT_DOWN_TILED) != 0;
  const bool block_major = down_tiled ||
                           ((w->down_row_stride == 0 || w->down_row_stride == 16) &&
                            (w->down_absmax_row_stride == 0 || w->down_absmax_row_stride == 1) &&
                            w->down_absmax_pair == 0);
  NSM_REQUIRE(block_major, NSM_ERR_UNSUPPORTED, "cache pools must use the block-major or tiled down layout");
  if (n <= 0) return NSM_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  PromoteParams p{};
  p.gate = const_cast<uint8_t*>(w->gate_packed);
  p.gate_am = const_cast<float*>(w->gate_absmax);
  p.up = const_cast<uint8_t*>(w->up_packed);
  p.up_am = const_cast<float*>(w->up_absmax);
  p.down = const_cast<uint8_t*>(w->down_packed);
  p.down_am = const_cast<float*>(w->down_absmax);
  p.gstride = w->gateup_block_stride ? w->gateup_block_stride : (int64_t)16 * hidden;
  p.gastride = w->gateup_absmax_block_stride ? w->gateup_absmax_block_stride : (int64_t)hidden / 2;
  p.dbs = w->down_block_stride ? w->down_block_stride : (int64_t)16 * hidden;
  p.dabs = w->down_absmax_block_stride ? w->down_absmax_block_stride : hidden;
  p.H = hidden;
  p.src = src_rows;
  p.dst = dst_rows;
  dim3 grid(16, n);
  cache_promote_copy_kernel<<<grid, 256, 0, s>>>(p);
  NSM_CHECK_CUDA(cudaGetLastError());
  cache_table_update_kernel<<<1, 32, 0, s>>>(block_ids, evicted_ids, dst_rows, n, slot_of_block);
  NSM_CHECK_CUDA(cudaGetLastError());
  return NSM_OK;
}

}  // extern "C"
