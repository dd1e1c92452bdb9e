// saga_atopn_decode_noalloc: the steady-state decode step for callers that
// cannot hand the library a workspace. Some hosts may not allocate device
// memory once they are running: an inference server that reserved all of the
// GPU's memory at start-up, a caching allocator the caller does not want
// fragmented by a small per-shape buffer, or a plugin interface whose decode
// hook receives tensors but no allocator. This entry point keeps the fused
// kernel's scratch (control counters and exchange slots) in a fixed array in
// the library's own device memory instead.
//
// Limits, stated once:
//   * The scratch holds kStaticScratchBytes (8 MiB). Shapes whose
//     saga_workspace_bytes(args, SAGA_OP_ATOPN_DECODE) exceeds it are refused
//     with SAGA_ERR_WORKSPACE; use saga_atopn_decode with a caller workspace.
//   * There is one scratch per device. Calls on the same device that overlap
//     on the GPU (different streams, or different host threads) race on it and
//     produce wrong results; serialise them.
//   * Each call first zero-fills the bytes it uses (one cudaMemsetAsync on the
//     caller's stream), because the previous call may have used other shapes.
//   * The first call on a device looks up the array's address through the
//     runtime; make that first call outside any stream capture.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/saga_b200.h"

namespace saga {
int abi_fail(int code, const std::string& msg);  // sets saga_last_error (abi.cu)
}

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_scratch[kStaticScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of this device's copy of g_scratch (looked up once).
int scratch_of(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return saga::abi_fail(SAGA_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return saga::abi_fail(SAGA_ERR_UNSUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p)
      return saga::abi_fail(SAGA_ERR_CUDA, std::string("cudaGetSymbolAddress of the static scratch: ") +
                                               cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return SAGA_OK;
}

}  // namespace

extern "C" {

size_t saga_noalloc_scratch_bytes(void) { return kStaticScratchBytes; }

int saga_atopn_decode_noalloc(const SagaAttnArgs* args, void* stream) {
  if (!args) return saga::abi_fail(SAGA_ERR_INVALID, "args is NULL");
  const size_t need = saga_workspace_bytes(args, SAGA_OP_ATOPN_DECODE);
  if (need == 0) return SAGA_ERR_INVALID;  // saga_workspace_bytes set the message
  if (need > kStaticScratchBytes)
    return saga::abi_fail(SAGA_ERR_WORKSPACE,
                          "these shapes need " + std::to_string(need) + " bytes of scratch; the static scratch of "
                          "saga_atopn_decode_noalloc holds " + std::to_string(kStaticScratchBytes) +
                          " (use saga_atopn_decode with a caller workspace)");
  void* scratch = nullptr;
  int rc = scratch_of(&scratch);
  if (rc) return rc;
  if (args->B > 0) {
    cudaError_t e = cudaMemsetAsync(scratch, 0, need, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess)
      return saga::abi_fail(SAGA_ERR_CUDA, std::string("clearing the static scratch: ") + cudaGetErrorString(e));
  }
  SagaAttnArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kStaticScratchBytes;
  return saga_atopn_decode(&a, stream);
}

}  // extern "C"
