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
//   * The array is part of the library's device image: every CUDA context
//     that loads libsaga_b200.so holds its 8 MiB until exit, whether or not
//     this entry point is ever called.
//   * There is one scratch per device. Calls on the same device that overlap
//     on the GPU (different streams, or different host threads) race on it and
//     produce wrong results; serialise them.
//   * Sequence sharding (shards > 1) is refused: the other devices would need
//     this device's scratch mapped as their peer workspace, which a caller
//     cannot arrange without an address.
//   * A call is validated completely before it touches the scratch; then it
//     zero-fills the bytes it uses (one cudaMemsetAsync on the caller's
//     stream), because the previous call may have used other shapes.
//   * Every call looks the array's address up through the runtime (no cached
//     pointer survives a device reset). The first call on a device may load
//     the library's device code there; make that first call outside any stream
//     capture.
// No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <string>

#include "../../include/saga_b200.h"

namespace saga {
int abi_fail(int code, const std::string& msg);          // sets saga_last_error (abi.cu)
int abi_check(const SagaAttnArgs* a, int op);            // host validation (abi.cu)
}

namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_scratch[kStaticScratchBytes];

// Device address of the current device's copy of g_scratch.
int scratch_of(void** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
  if (e != cudaSuccess || !p)
    return saga::abi_fail(SAGA_ERR_CUDA,
                          std::string("cudaGetSymbolAddress of the static scratch: ") + cudaGetErrorString(e));
  *out = p;
  return SAGA_OK;
}

}  // namespace

extern "C" {

size_t saga_noalloc_scratch_bytes(void) { return kStaticScratchBytes; }

int saga_atopn_decode_noalloc(const SagaAttnArgs* args, void* stream) {
  if (!args) return saga::abi_fail(SAGA_ERR_INVALID, "args is NULL");
  if (args->shards > 1)
    return saga::abi_fail(SAGA_ERR_UNSUPPORTED,
                          "saga_atopn_decode_noalloc does not support sequence sharding (shards > 1); "
                          "use saga_atopn_decode with mapped shard workspaces");
  int rc = saga::abi_check(args, SAGA_OP_ATOPN_DECODE);
  if (rc) return rc;  // abi_check set the message; the scratch is untouched
  const size_t need = saga_workspace_bytes(args, SAGA_OP_ATOPN_DECODE);
  if (need == 0) return SAGA_ERR_INVALID;  // saga_workspace_bytes set the message
  if (need > kStaticScratchBytes)
    return saga::abi_fail(SAGA_ERR_WORKSPACE,
                          "these shapes need " + std::to_string(need) + " bytes of scratch; the static scratch of "
                          "saga_atopn_decode_noalloc holds " + std::to_string(kStaticScratchBytes) +
                          " (use saga_atopn_decode with a caller workspace)");
  if (args->B == 0) return saga_atopn_decode(args, stream);  // nothing to launch
  void* scratch = nullptr;
  rc = scratch_of(&scratch);
  if (rc) return rc;
  cudaError_t e = cudaMemsetAsync(scratch, 0, need, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return saga::abi_fail(SAGA_ERR_CUDA, std::string("clearing the static scratch: ") + cudaGetErrorString(e));
  SagaAttnArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kStaticScratchBytes;
  return saga_atopn_decode(&a, stream);
}

}  // extern "C"
