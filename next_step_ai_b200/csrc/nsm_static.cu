// nsm_static.cu -- nsm_decode_gathered_static: the gathered-block decode MLP
// with its scratch in a file-scope device array instead of a caller-owned
// workspace.
//
// Some callers cannot allocate device memory at the point where they decode:
// code running under an allocator that must not grow (a fixed memory pool
// handed out before serving starts), a host language binding that has no
// access to the CUDA allocator, or a plug-in that is not allowed to own
// device memory.  For them this entry point allocates nothing: its scratch is
// `g_static_scratch` below, a fixed array that the CUDA runtime places on each
// device when it loads this file's module there, and that stays there until
// the process exits.
//
// Limits: hidden <= NSM_STATIC_MAX_HIDDEN (16384) and num_blocks_gathered <=
// NSM_STATIC_MAX_BLOCKS (256); the scratch for the largest such call is
// 6,423,296 bytes (the decode workspace layout at those limits, checked by a
// host test through nsm_decode_rows_workspace_bytes), so the array is 6.5 MiB.
//
// Every call on a device shares the one array and finds the previous call's
// contents in it.  The parts that must start at zero (the reduction tickets at
// the head of the workspace layout) are cleared with a stream-ordered memset at
// the start of each call; everything else is written before it is read.  The
// device error word in that head is NOT cleared by a call: a kernel that gave
// up on a bounded wait records NSM_ERR_TIMEOUT there, and it stays until
// nsm_static_error reads and clears it.  Calls whose GPU work overlaps
// (different streams, different host threads without ordering between their
// streams) race on the array and give wrong results.
//
// Set-up: the first call on a device, with that device current, looks up the
// array's device address with cudaGetSymbolAddress (which also makes the
// runtime load this module on that device) and caches it.  Make that first
// call before any stream capture on the device.  The cached address does not
// survive cudaDeviceReset (the module is loaded again, possibly elsewhere):
// do not use this entry point on a device after resetting it.
#include <cuda_runtime.h>

#include <mutex>

#include "nsm.h"
#include "nsm_internal.h"

namespace nsm {
namespace {

constexpr size_t kStaticScratchBytes = (size_t)13 << 19;  // 6.5 MiB

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

int static_scratch_for(int device, void** out) {
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (g_static_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_static_scratch)");
    if (p == nullptr) return fail(NSM_ERR_CUDA, "cudaGetSymbolAddress(g_static_scratch) returned NULL");
    g_static_ptr[device] = p;
  }
  *out = g_static_ptr[device];
  return NSM_OK;
}

}  // namespace
}  // namespace nsm

using namespace nsm;

extern "C" int nsm_decode_gathered_static(const void* x, int32_t x_dtype, int32_t hidden,
                                          int32_t num_blocks_gathered, const nsm_mlp_weights* w, void* y,
                                          int32_t y_dtype, float* act_out, nsm_stream_t stream) {
  NSM_REQUIRE(hidden > 0 && hidden <= NSM_STATIC_MAX_HIDDEN, NSM_ERR_UNSUPPORTED,
              "nsm_decode_gathered_static: hidden must be in [1, 16384] (the static scratch limit); "
              "use nsm_decode_gathered with a caller workspace for larger shapes");
  NSM_REQUIRE(num_blocks_gathered > 0 && num_blocks_gathered <= NSM_STATIC_MAX_BLOCKS, NSM_ERR_UNSUPPORTED,
              "nsm_decode_gathered_static: num_blocks_gathered must be in [1, 256] (the static scratch limit); "
              "use nsm_decode_gathered with a caller workspace for more blocks");
  int dev = -1;
  NSM_CHECK_CUDA(cudaGetDevice(&dev));
  NSM_REQUIRE(dev >= 0 && dev < kMaxDevices, NSM_ERR_DEVICE, "device index out of range");
  void* scratch = nullptr;
  int st = static_scratch_for(dev, &scratch);
  if (st) return st;
  const int I = 64 * ((num_blocks_gathered * 32 + 63) / 64);
  const size_t need = decode_ws_layout(nullptr, hidden, I, num_blocks_gathered, 1).bytes;
  NSM_REQUIRE(need <= kStaticScratchBytes, NSM_ERR_WORKSPACE,
              "nsm_decode_gathered_static: shape needs more scratch than the static array holds");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // The tickets at the head of the layout must read zero when the kernels
  // start; a call that failed part-way may have left them non-zero.  The
  // error word between them keeps a timeout of an earlier call for
  // nsm_static_error.
  char* head = reinterpret_cast<char*>(scratch);
  const size_t err_off = (size_t)(reinterpret_cast<char*>(decode_ws_layout(scratch, 64, 64, 1, 1).err) - head);
  NSM_CHECK_CUDA(cudaMemsetAsync(head, 0, err_off, s));
  NSM_CHECK_CUDA(cudaMemsetAsync(head + err_off + sizeof(int), 0,
                                 align_up((size_t)kCounterInts * sizeof(int), 256) - err_off - sizeof(int), s));
  return nsm_decode_gathered(x, x_dtype, hidden, num_blocks_gathered, w, y, y_dtype, act_out, scratch,
                             kStaticScratchBytes, s);
}

extern "C" int nsm_static_error(int32_t* code_out, nsm_stream_t stream) {
  NSM_REQUIRE(code_out != nullptr, NSM_ERR_INVALID_ARG, "nsm_static_error: code_out is NULL");
  int dev = -1;
  NSM_CHECK_CUDA(cudaGetDevice(&dev));
  NSM_REQUIRE(dev >= 0 && dev < kMaxDevices, NSM_ERR_DEVICE, "device index out of range");
  void* scratch = nullptr;
  int st = static_scratch_for(dev, &scratch);
  if (st) return st;
  int* err = decode_ws_layout(scratch, 64, 64, 1, 1).err;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int32_t v = 0;
  NSM_CHECK_CUDA(cudaMemcpyAsync(&v, err, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  NSM_CHECK_CUDA(cudaMemsetAsync(err, 0, sizeof(int32_t), s));
  NSM_CHECK_CUDA(cudaStreamSynchronize(s));
  *code_out = v;
  return NSM_OK;
}
