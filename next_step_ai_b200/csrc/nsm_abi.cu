// nsm_abi.cu -- status strings, per-thread error detail, device checks and the
// decode workspace layout.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <mutex>
#include <algorithm>
#include <string>

#include "nsm_internal.h"

namespace nsm {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  g_last_error = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return NSM_ERR_CUDA;
}

static std::atomic<int> g_copy_wait_spins{kDefaultCopyWaitSpins};
int copy_wait_spins() { return g_copy_wait_spins.load(std::memory_order_relaxed); }

static std::mutex g_dev_mu;
static DeviceInfo g_dev_cache[64];

int current_device(DeviceInfo* info) {
  int dev = -1;
  NSM_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(NSM_ERR_DEVICE, "device index out of range");
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_dev_cache[dev].device == dev) {
      *info = g_dev_cache[dev];
      return NSM_OK;
    }
  }
  DeviceInfo d;
  d.device = dev;
  NSM_CHECK_CUDA(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
  NSM_CHECK_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
  NSM_CHECK_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
  NSM_CHECK_CUDA(cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  if (d.major != 10 || d.minor != 0) {
    char buf[128];
    snprintf(buf, sizeof(buf), "this library is built for sm_100a (B200); device %d is sm_%d%d", dev, d.major,
             d.minor);
    return fail(NSM_ERR_DEVICE, buf);
  }
  std::lock_guard<std::mutex> lk(g_dev_mu);
  g_dev_cache[dev] = d;
  *info = d;
  return NSM_OK;
}

DecodeWs decode_ws_layout(void* base, int hidden, int intermediate, int top_k, int rank, int rows) {
  DecodeWs w{};
  char* b = reinterpret_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = b ? b + off : nullptr;
    off = align_up(off + bytes, 256);
    return p;
  };
  const int nb = intermediate / 32;
  int* tick = reinterpret_cast<int*>(take((size_t)kCounterInts * sizeof(int)));
  w.ticket_router_a = tick;
  w.err = tick ? tick + 2 : nullptr;
  w.down_meta = tick ? tick + 3 : nullptr;
  w.count = tick ? tick + 5 : nullptr;
  // the gate/up kernel's per-block tickets return to zero within a call, so
  // they live in the head too, where every shape finds them zero
  static_assert(8 + kMaxTopK <= kCounterInts, "gate/up tickets in the counter head");
  w.gu_ticket = tick ? reinterpret_cast<unsigned*>(tick + 8) : nullptr;
  // the down partials sit at a fixed offset too: a layer's pending output is
  // read by the next call, whose router may have a different k or rank
  w.ypart = reinterpret_cast<float*>(take((size_t)kMaxSlotGroups * hidden * sizeof(float)));
  // router scratch: one copy per routed row (multi-row routing)
  const size_t R = (size_t)std::max(1, rows);
  w.latent_part = reinterpret_cast<float*>(take(R * kRouterMaxCtas * rank * sizeof(float)));
  w.sumsq_part = reinterpret_cast<float*>(take(R * kRouterMaxCtas * sizeof(float)));
  w.latent = reinterpret_cast<float*>(take(R * rank * sizeof(float)));
  w.norm_scale = reinterpret_cast<float*>(take(sizeof(float)));
  w.scores = reinterpret_cast<float*>(take(R * nb * sizeof(float)));
  w.x16 = reinterpret_cast<__half*>(take((size_t)hidden * sizeof(__half)));
  w.x16lo = reinterpret_cast<__half*>(take((size_t)hidden * sizeof(__half)));
  w.xscale = reinterpret_cast<float*>(take((size_t)(hidden / 64) * sizeof(float)));
  w.rows = reinterpret_cast<int*>(take((size_t)top_k * sizeof(int)));
  w.sel_idx = reinterpret_cast<int*>(take(R * top_k * sizeof(int)));
  w.row_block = reinterpret_cast<int*>(take((size_t)top_k * sizeof(int)));
  w.gu_part = reinterpret_cast<float*>(take((size_t)top_k * kMaxUnitsPerSlot * 64 * sizeof(float)));
  w.act16 = reinterpret_cast<__half*>(take((size_t)top_k * 32 * sizeof(__half)));
  w.act16lo = reinterpret_cast<__half*>(take((size_t)top_k * 32 * sizeof(__half)));
  w.act_scale = reinterpret_cast<float*>(take((size_t)top_k * sizeof(float)));
  w.bytes = off;
  return w;
}

}  // namespace nsm

using namespace nsm;

extern "C" {

int nsm_abi_version(void) { return 4; }

const char* nsm_status_string(int status) {
  switch (status) {
    case NSM_OK: return "ok";
    case NSM_ERR_INVALID_ARG: return "invalid argument";
    case NSM_ERR_UNSUPPORTED: return "unsupported shape";
    case NSM_ERR_CUDA: return "CUDA error";
    case NSM_ERR_TIMEOUT: return "device wait timed out";
    case NSM_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case NSM_ERR_DEVICE: return "unsupported device";
    default: return "unknown status";
  }
}

const char* nsm_last_error(void) { return g_last_error.c_str(); }

int nsm_workspace_init(void* ws, size_t ws_bytes, nsm_stream_t stream) {
  if (ws == nullptr || ws_bytes == 0) return fail(NSM_ERR_WORKSPACE, "nsm_workspace_init: empty workspace");
  NSM_CHECK_CUDA(cudaMemsetAsync(ws, 0, ws_bytes, reinterpret_cast<cudaStream_t>(stream)));
  return NSM_OK;
}

int nsm_workspace_error(void* ws, size_t ws_bytes, int32_t* code_out, nsm_stream_t stream) {
  if (code_out == nullptr) return fail(NSM_ERR_INVALID_ARG, "nsm_workspace_error: code_out is NULL");
  if (ws == nullptr || ws_bytes < (size_t)kCounterInts * sizeof(int))
    return fail(NSM_ERR_WORKSPACE, "nsm_workspace_error: workspace missing or too small");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* err = decode_ws_layout(ws, 64, 64, 1, 1).err;
  int32_t v = 0;
  NSM_CHECK_CUDA(cudaMemcpyAsync(&v, err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  NSM_CHECK_CUDA(cudaMemsetAsync(err, 0, sizeof(int32_t), s));
  NSM_CHECK_CUDA(cudaStreamSynchronize(s));
  *code_out = v;
  return NSM_OK;
}

int nsm_set_copy_wait_limit(int32_t spins) {
  if (spins < 0) return fail(NSM_ERR_INVALID_ARG, "nsm_set_copy_wait_limit: spins must be >= 0 (0 = the default)");
  const int prev = g_copy_wait_spins.exchange(spins > 0 ? spins : kDefaultCopyWaitSpins);
  return prev;
}

int nsm_workspace_selection(const void* ws, size_t ws_bytes, int32_t hidden, int32_t intermediate, int32_t top_k,
                            int32_t rank, int32_t* blocks_out, int32_t* count_out, nsm_stream_t stream) {
  if (blocks_out == nullptr || count_out == nullptr)
    return fail(NSM_ERR_INVALID_ARG, "nsm_workspace_selection: blocks_out / count_out is NULL");
  if (hidden <= 0 || hidden % 64 != 0 || intermediate <= 0 || intermediate % 64 != 0 || top_k <= 0 || rank <= 0)
    return fail(NSM_ERR_INVALID_ARG, "nsm_workspace_selection: bad shape");
  const int k = std::min(top_k, intermediate / 32);
  const DecodeWs need = decode_ws_layout(nullptr, hidden, intermediate, k, rank);
  if (ws == nullptr || ws_bytes < need.bytes)
    return fail(NSM_ERR_WORKSPACE, "nsm_workspace_selection: workspace missing or smaller than the decode layout");
  const DecodeWs w = decode_ws_layout(const_cast<void*>(ws), hidden, intermediate, k, rank);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  NSM_CHECK_CUDA(cudaMemcpyAsync(blocks_out, w.row_block, (size_t)k * sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
  NSM_CHECK_CUDA(cudaMemcpyAsync(count_out, w.count, sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
  return NSM_OK;
}

size_t nsm_decode_workspace_bytes(int hidden, int intermediate, int top_k, int rank) {
  if (hidden <= 0 || intermediate <= 0 || top_k <= 0 || rank <= 0) return 0;
  return decode_ws_layout(nullptr, hidden, intermediate, top_k, rank).bytes;
}

size_t nsm_route_workspace_bytes(int hidden, int num_blocks, int top_k, int rank, int rows) {
  if (hidden <= 0 || num_blocks <= 0 || top_k <= 0 || rank <= 0 || rows <= 0) return 0;
  return decode_ws_layout(nullptr, hidden, num_blocks * 32, top_k, rank, rows).bytes;
}

}  // extern "C"
