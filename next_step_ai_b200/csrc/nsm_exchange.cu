// nsm_exchange.cu -- per-rank exchange buffers for the fused cross-GPU sum of a
// layer's output (see ExchangeDev in nsm_internal.h).  Buffers are plain
// cudaMalloc allocations shared between the processes of one node with CUDA
// IPC handles; peers are reached with ordinary loads and stores over NVLink
// (no multicast objects).
#include <cuda_runtime.h>

#include <cstring>
#include <new>

#include "nsm.h"
#include "nsm_internal.h"

namespace nsm {

struct ExchangeHost {
  ExchangeDev dev{};
  void* local = nullptr;                // this rank's buffer
  void* peers[kMaxWorld] = {};          // opened IPC mappings (nullptr for self)
  size_t bytes = 0;
  int device = -1;
};

static size_t exchange_data_off() { return 256; }
static size_t exchange_total(int world, int hidden) {
  return exchange_data_off() + (size_t)2 * world * hidden * sizeof(unsigned long long);
}

}  // namespace nsm

using namespace nsm;

extern "C" {

size_t nsm_exchange_bytes(int world, int hidden) {
  if (world <= 0 || world > kMaxWorld || hidden <= 0) return 0;
  return exchange_total(world, hidden);
}

int nsm_exchange_create(int32_t world, int32_t rank, int32_t hidden, nsm_exchange** ex_out, void* ipc_handle_out) {
  NSM_REQUIRE(ex_out != nullptr && ipc_handle_out != nullptr, NSM_ERR_INVALID_ARG, "NULL pointer");
  NSM_REQUIRE(world >= 1 && world <= kMaxWorld, NSM_ERR_UNSUPPORTED, "world must be in [1, 8]");
  NSM_REQUIRE(rank >= 0 && rank < world, NSM_ERR_INVALID_ARG, "rank out of range");
  NSM_REQUIRE(hidden > 0 && hidden % 64 == 0 && hidden <= kMaxHidden, NSM_ERR_UNSUPPORTED, "bad hidden size");
  ExchangeHost* h = new (std::nothrow) ExchangeHost();
  NSM_REQUIRE(h != nullptr, NSM_ERR_INVALID_ARG, "out of host memory");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) {
    h->device = dev;
    h->bytes = exchange_total(world, hidden);
    e = cudaMalloc(&h->local, h->bytes);
  }
  if (e == cudaSuccess) e = cudaMemset(h->local, 0, h->bytes);
  cudaIpcMemHandle_t handle;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&handle, h->local);
  if (e != cudaSuccess) {
    if (h->local) cudaFree(h->local);
    delete h;
    return cuda_fail(e, "nsm_exchange_create");
  }
  std::memcpy(ipc_handle_out, &handle, sizeof(handle));
  h->dev.world = world;
  h->dev.rank = rank;
  h->dev.hidden = hidden;
  h->dev.spin_limit = kDefaultExchangeSpins;
  h->dev.counter = reinterpret_cast<uint32_t*>(h->local);
  *ex_out = reinterpret_cast<nsm_exchange*>(h);
  return NSM_OK;
}

int nsm_exchange_connect(nsm_exchange* ex, const void* handles) {
  NSM_REQUIRE(ex != nullptr && handles != nullptr, NSM_ERR_INVALID_ARG, "NULL pointer");
  ExchangeHost* h = reinterpret_cast<ExchangeHost*>(ex);
  const int world = h->dev.world;
  for (int p = 0; p < world; ++p) {
    char* base;
    if (p == h->dev.rank) {
      base = reinterpret_cast<char*>(h->local);
    } else {
      cudaIpcMemHandle_t handle;
      std::memcpy(&handle, reinterpret_cast<const char*>(handles) + (size_t)p * NSM_IPC_HANDLE_BYTES, sizeof(handle));
      void* ptr = nullptr;
      NSM_CHECK_CUDA(cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess));
      h->peers[p] = ptr;
      base = reinterpret_cast<char*>(ptr);
    }
    h->dev.data[p] = reinterpret_cast<unsigned long long*>(base + exchange_data_off());
  }
  return NSM_OK;
}

int nsm_exchange_connect_local(nsm_exchange* const* exs, int32_t n) {
  NSM_REQUIRE(exs != nullptr && n >= 1 && n <= kMaxWorld, NSM_ERR_INVALID_ARG, "need 1..8 exchanges");
  const ExchangeHost* first = reinterpret_cast<const ExchangeHost*>(exs[0]);
  NSM_REQUIRE(first != nullptr && first->dev.world == n, NSM_ERR_INVALID_ARG, "exchange world != n");
  for (int i = 0; i < n; ++i) {
    const ExchangeHost* h = reinterpret_cast<const ExchangeHost*>(exs[i]);
    NSM_REQUIRE(h != nullptr && h->dev.world == n && h->dev.rank == i && h->dev.hidden == first->dev.hidden,
                NSM_ERR_INVALID_ARG, "exchanges must be ranks 0..n-1 of one world with one hidden size");
  }
  for (int i = 0; i < n; ++i) {
    ExchangeHost* h = reinterpret_cast<ExchangeHost*>(exs[i]);
    for (int p = 0; p < n; ++p) {
      char* base = reinterpret_cast<char*>(reinterpret_cast<const ExchangeHost*>(exs[p])->local);
      h->dev.data[p] = reinterpret_cast<unsigned long long*>(base + exchange_data_off());
    }
  }
  return NSM_OK;
}

int nsm_exchange_set_spin_limit(nsm_exchange* ex, int32_t spins) {
  NSM_REQUIRE(ex != nullptr, NSM_ERR_INVALID_ARG, "NULL exchange");
  NSM_REQUIRE(spins >= 0, NSM_ERR_INVALID_ARG, "spins must be >= 0 (0 = the default)");
  reinterpret_cast<ExchangeHost*>(ex)->dev.spin_limit = spins > 0 ? spins : kDefaultExchangeSpins;
  return NSM_OK;
}

int nsm_exchange_destroy(nsm_exchange* ex) {
  if (ex == nullptr) return NSM_OK;
  ExchangeHost* h = reinterpret_cast<ExchangeHost*>(ex);
  for (int p = 0; p < kMaxWorld; ++p)
    if (h->peers[p]) cudaIpcCloseMemHandle(h->peers[p]);
  if (h->local) cudaFree(h->local);
  delete h;
  return NSM_OK;
}

}  // extern "C"

namespace nsm {
const ExchangeDev* exchange_dev(const nsm_exchange* ex) {
  return ex ? &reinterpret_cast<const ExchangeHost*>(ex)->dev : nullptr;
}
}  // namespace nsm
