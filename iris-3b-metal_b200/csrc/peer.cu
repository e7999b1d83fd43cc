// Peer memory for sequence parallelism across processes, one per GPU:
//   * CUDA IPC export / import of the buffers that other ranks' kernels write
//     into (the full-sequence attention operands, the output token rows, the
//     barrier flags), so a producing kernel can store straight into the
//     consumer's buffer over NVLink;
//   * a signal-and-wait barrier on flags in peer memory, with bounded waits.
// The reference runs on one device; this has no counterpart there.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "iris_abi_internal.h"

namespace iris {
namespace peer {

constexpr int MAX_PEERS = IRIS_MAX_PEERS;

struct PeerFlags {
  unsigned int* flags[MAX_PEERS];  // rank j's flag array, mapped into this process
};

IRIS_DEVICE void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

IRIS_DEVICE unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread j (j != rank) writes `epoch` into slot `rank` of rank j's flags, then
// waits until rank j has written at least `epoch` into slot j of this rank's
// flags. Every write this rank's stream issued before this kernel (the
// producing kernel's peer stores) completed before it started; the fence and
// the release store order them before the flag for the peer that acquires it.
// A wait that outlasts `timeout_ns` records kErrWaitTimeout and gives up.
__global__ void barrier_kernel(unsigned int* __restrict__ flags, PeerFlags peers, int rank, int world,
                               unsigned int epoch, uint64_t timeout_ns) {
  const int j = threadIdx.x;
  if (j >= world || j == rank) return;
  __threadfence_system();
  st_release_sys(peers.flags[j] + rank, epoch);
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (static_cast<int>(ld_acquire_sys(flags + j) - epoch) >= 0) return;
    if ((i & 15u) == 15u && global_timer_ns() - t0 > timeout_ns) {
      atomicOr(&g_device_error, kErrWaitTimeout);
      return;
    }
    __nanosleep(64);
  }
}

PFN_cuMemGetAddressRange_v3020 range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  });
  return fn;
}

}  // namespace peer
}  // namespace iris

using namespace iris;

extern "C" int iris_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  IRIS_REQUIRE(ptr && handle && offset, "ipc_export: null pointer");
  auto fn = peer::range_fn();
  IRIS_REQUIRE(fn != nullptr, "ipc_export: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return set_error(IRIS_ECUDA, "ipc_export: cuMemGetAddressRange failed (%d)", static_cast<int>(r));
  cudaIpcMemHandle_t h;
  IRIS_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(h) == IRIS_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return IRIS_OK;
}

extern "C" int iris_ipc_import(const void* handle, void** base) {
  IRIS_REQUIRE(handle && base, "ipc_import: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  IRIS_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
  return IRIS_OK;
}

extern "C" int iris_ipc_close(void* base) {
  IRIS_REQUIRE(base, "ipc_close: null pointer");
  IRIS_CUDA(cudaIpcCloseMemHandle(base));
  return IRIS_OK;
}

extern "C" int iris_peer_barrier(unsigned int* flags, void* const* peer_flags, int rank, int world,
                                 unsigned int epoch, int64_t timeout_ns, void* stream) {
  IRIS_REQUIRE(flags && peer_flags, "peer_barrier: null pointer");
  IRIS_REQUIRE(world >= 1 && world <= IRIS_MAX_PEERS && rank >= 0 && rank < world, "peer_barrier: bad rank / world");
  IRIS_REQUIRE(timeout_ns > 0, "peer_barrier: timeout must be positive");
  IRIS_REQUIRE(aligned_n(flags, 4), "peer_barrier: flags must be 4-byte aligned");
  peer::PeerFlags pf{};
  for (int j = 0; j < world; ++j) {
    IRIS_REQUIRE(j == rank || (peer_flags[j] != nullptr && aligned_n(peer_flags[j], 4)), "peer_barrier: peer flags");
    pf.flags[j] = static_cast<unsigned int*>(peer_flags[j]);
  }
  if (world == 1) return IRIS_OK;
  peer::barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, pf, rank, world, epoch,
                                                                        static_cast<uint64_t>(timeout_ns));
  IRIS_CUDA(cudaGetLastError());
  return IRIS_OK;
}
