// nsm_internal.h -- host-side helpers shared by the ABI translation units:
// error reporting, device checks, and the decode workspace layout.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/nsm.h"

namespace nsm {

// Thread-local detail for nsm_last_error().
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define NSM_CHECK_CUDA(expr)                         \
  do {                                               \
    cudaError_t _e = (expr);                         \
    if (_e != cudaSuccess) return cuda_fail(_e, #expr); \
  } while (0)

#define NSM_REQUIRE(cond, status, msg) \
  do {                                 \
    if (!(cond)) return fail((status), (msg)); \
  } while (0)

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int major = 0, minor = 0;
  int max_smem_optin = 0;
};
// Current device's properties (cached per device); status != 0 if not sm_100.
int current_device(DeviceInfo* info);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Limits of the single-token decode path.
constexpr int kMaxRank = 256;
constexpr int kMaxTopK = 4096;
constexpr int kMaxNumBlocks = 8192;     // top-k sort capacity of the router
constexpr int kMaxUnitsPerSlot = 64;    // gate/up column splits per block
constexpr int kMaxSlotGroups = 32;      // down split-K groups
constexpr int kRouterMaxCtas = 256;
constexpr int kMaxHidden = 65536;       // counters are sized for this
constexpr int kCounterInts = 2 + kMaxTopK + kMaxHidden / 32;

// Decode workspace: one contiguous caller-owned buffer, 256-byte aligned parts.
// Cross-GPU exchange of a layer's output (device view of nsm_exchange).
// Rank r's buffer: counter (epoch of the last completed exchange) | data
// [2 slots][world][H] 8-byte words (fp32 value bits | epoch << 32; slot =
// epoch & 1).  Every rank stores its chunk of the layer output into every
// rank's buffer and sums the ranks' words in rank order once each carries the
// current epoch.
constexpr int kMaxWorld = 8;
// Default bounds of the device waits: polls of a peer's exchange words, and
// tries of a warp's bulk-copy mbarrier.  Both are runtime settings
// (nsm_exchange_set_spin_limit, nsm_set_copy_wait_limit).
constexpr int kDefaultExchangeSpins = 1 << 24;
constexpr int kDefaultCopyWaitSpins = 1 << 22;
int copy_wait_spins();
struct ExchangeDev {
  unsigned long long* data[kMaxWorld];  // peer p's data region (mapped into this process)
  uint32_t* counter;                    // this rank's epoch counter
  int world;
  int rank;
  int hidden;
  int spin_limit;                       // polls of one peer word before NSM_ERR_TIMEOUT
};

const ExchangeDev* exchange_dev(const nsm_exchange* ex);

struct DecodeWs {
  // counters (must be zero between calls)
  int* ticket_router_a;          // [1] (head int 1 is unused)
  int* err;                      // [1] device-side error code (0 = none), sticky
  int* down_meta;                // [2] last down launch: total warps, log2 rows per reduction group
  // (count below and ypart live at fixed offsets after the counter head)
  // router
  float* latent_part;            // [kRouterMaxCtas][rank]
  float* sumsq_part;             // [kRouterMaxCtas]
  float* latent;                 // [rank]
  float* norm_scale;             // [1]
  float* scores;                 // [NB]
  // activations
  __half* x16;                   // [H] x / xscale rounded to fp16
  __half* x16lo;                 // [H] x / xscale - x16 rounded to fp16 (the hi + lo pair carries 22 bits)
  float* xscale;                 // [H/64]
  int* rows;                     // [top_k]
  int* count;                    // [1]
  int* sel_idx;                  // [top_k] router selection (when no idx_out)
  int* row_block;                // [top_k] block id of each compacted pool row
  float* gu_part;                // [top_k][kMaxUnitsPerSlot][2][32]
  unsigned* gu_ticket;           // [kMaxTopK] units of each block counted so far (counter head; zero between calls)
  __half* act16;                 // [top_k][32] SiLU(gate)*up / act_scale rounded to fp16
  __half* act16lo;               // [top_k][32] its remainder rounded to fp16
  float* act_scale;              // [top_k]
  float* ypart;                  // [kMaxSlotGroups][H]
  size_t bytes;
};

// Counters sit at fixed offsets at the head of every workspace, whatever the
// shape, so a zeroed workspace stays valid across calls with different shapes.
DecodeWs decode_ws_layout(void* base, int hidden, int intermediate, int top_k, int rank, int rows = 1);

// Cached occupancy-derived persistent grid sizes.
struct LaunchShape {
  int gateup_ctas = 0;
  int down_ctas = 0;
  int warps_per_cta = 8;
};
int launch_shape(LaunchShape* s);

// Launch with programmatic stream serialization (PDL): the kernel may begin
// before its predecessor finishes and must call griddepcontrol.wait before it
// reads the predecessor's results.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace nsm
