// extern "C" entry points of libsaga_b200.so: argument validation, then the
// launchers. Invalid requests are rejected on the host so that no kernel is
// ever launched on arguments it cannot handle.
#include <cuda.h>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/saga_b200.h"
#include "decode_internal.h"
#include "ops_internal.h"

namespace {

thread_local std::string g_err;
thread_local std::string g_launched;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

bool is_fp(int dt) { return dt == SAGA_BF16 || dt == SAGA_FP16 || dt == SAGA_FP32; }
int esz(int dt) { return dt == SAGA_FP32 ? 4 : 2; }
bool aligned(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shape, dtype and stride validation shared by the attention entry points.
int check_shapes(const SagaAttnArgs* a) {
  if (!a) return fail(SAGA_ERR_INVALID, "args is NULL");
  if (!is_fp(a->dtype)) return fail(SAGA_ERR_INVALID, "dtype must be bf16, fp16 or fp32");
  if (a->B < 0 || a->Hq <= 0 || a->Hk <= 0 || a->Hv <= 0 || a->L <= 0)
    return fail(SAGA_ERR_INVALID, "B >= 0, Hq, Hk, Hv, L > 0 required");
  if (a->Hq % a->Hk) return fail(SAGA_ERR_INVALID, "Hq must be a multiple of Hk");
  if (a->Hq % a->Hv) return fail(SAGA_ERR_INVALID, "Hq must be a multiple of Hv");
  if (a->D != 64 && a->D != 128) return fail(SAGA_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (a->Hq / a->Hk > saga::kMaxG) return fail(SAGA_ERR_UNSUPPORTED, "more than 32 query heads per key head");
  const int e = esz(a->dtype);
  // 16-byte rows for the staged K loads and the vector loads of V
  if ((a->k_sl * e) % 16 || (a->k_sh * e) % 16 || (a->k_sb * e) % 16)
    return fail(SAGA_ERR_INVALID, "key cache strides must be multiples of 16 bytes");
  if ((a->v_sl * e) % 16 || (a->v_sh * e) % 16 || (a->v_sb * e) % 16)
    return fail(SAGA_ERR_INVALID, "value cache strides must be multiples of 16 bytes");
  if (a->k_sl < a->D || a->v_sl < a->D) return fail(SAGA_ERR_INVALID, "position stride below head_dim");
  if (a->mask && a->mask_dtype != SAGA_BOOL && a->mask_dtype != a->dtype)
    return fail(SAGA_ERR_UNSUPPORTED, "mask must be bool or the logits dtype");
  if (!(a->scaling == a->scaling)) return fail(SAGA_ERR_INVALID, "scaling is NaN");
  if (a->top_n < 0) return fail(SAGA_ERR_INVALID, "top_n must not be negative");
  if (a->page_table) {
    if (a->page_len < 128 || (a->page_len & (a->page_len - 1)))
      return fail(SAGA_ERR_INVALID, "page_len must be a power of two and at least 128");
    if (a->num_pages <= 0) return fail(SAGA_ERR_INVALID, "num_pages must be positive");
    if (a->pt_sb <= 0 || a->pt_sb * (int64_t)a->page_len < a->L)
      return fail(SAGA_ERR_INVALID, "page table rows must cover L positions (pt_sb * page_len >= L)");
    // a head's rows inside a page must not run into the next head's
    if ((a->Hk > 1 && (int64_t)(a->page_len - 1) * a->k_sl + a->D > a->k_sh) ||
        (a->Hv > 1 && (int64_t)(a->page_len - 1) * a->v_sl + a->D > a->v_sh))
      return fail(SAGA_ERR_INVALID, "a page's rows of one head overlap the next head");
    if (a->shards > 1) return fail(SAGA_ERR_UNSUPPORTED, "paged caches are not supported with sequence sharding");
  }
  return SAGA_OK;
}

// Full validation of one call.
int check_attn(const SagaAttnArgs* a, int op) {
  int rc = check_shapes(a);
  if (rc) return rc;
  if (!a->q || !a->k || !a->v) return fail(SAGA_ERR_INVALID, "q, k and v must be non-NULL");
  if (!aligned(a->k, 16) || !aligned(a->v, 16))
    return fail(SAGA_ERR_INVALID, "key and value caches must be 16-byte aligned");
  if (a->page_table && !aligned(a->page_table, 4)) return fail(SAGA_ERR_INVALID, "page_table must be 4-byte aligned");
  if (op == SAGA_OP_LOGITS) {
    if (!a->logits_out || a->lo_ld < a->L) return fail(SAGA_ERR_INVALID, "logits_out [R, >=L] required");
    return SAGA_OK;
  }
  if (!a->out) return fail(SAGA_ERR_INVALID, "out must be non-NULL");
  if (op == SAGA_OP_ATOPN_DECODE || op == SAGA_OP_ATOPN_CALIBRATE) {
    if (a->top_n <= 0) return fail(SAGA_ERR_INVALID, "top_n must be positive");
    if (op == SAGA_OP_ATOPN_DECODE && !a->thr_in) return fail(SAGA_ERR_INVALID, "thr_in required");
  }
  if (a->sel_idx_out && a->sel_ld <= 0) return fail(SAGA_ERR_INVALID, "sel_ld must be positive");
  if (a->nsel < 0 || a->nsel > a->L) return fail(SAGA_ERR_INVALID, "nsel outside [0, L]");
  if (a->nsel > 0 && a->nsel < a->L && a->L - a->nsel != 256)
    return fail(SAGA_ERR_INVALID, "positions past nsel must be exactly the 256-row tail replica");
  if (a->shards > 1) {
    if (a->shards > 8 || a->shard < 0 || a->shard >= a->shards)
      return fail(SAGA_ERR_INVALID, "shards in [1, 8] and 0 <= shard < shards required");
    if (op != SAGA_OP_ATOPN_DECODE && op != SAGA_OP_DENSE_DECODE && op != SAGA_OP_ATOPN_CALIBRATE)
      return fail(SAGA_ERR_UNSUPPORTED, "sequence sharding supports the decode, calibration and dense ops");
    if (a->dtype == SAGA_FP32 || a->Hq / a->Hk > 16)
      return fail(SAGA_ERR_UNSUPPORTED, "sequence sharding needs the tensor-core path (16-bit, G <= 16)");
    for (int s = 0; s < a->shards; ++s)
      if (!a->shard_workspaces[s]) return fail(SAGA_ERR_INVALID, "every shard workspace must be mapped");
    if (a->shard_workspaces[a->shard] != a->workspace)
      return fail(SAGA_ERR_INVALID, "shard_workspaces[shard] must be this call's workspace");
  }
  if (a->k_new || a->v_new) {
    if (!a->k_new || !a->v_new) return fail(SAGA_ERR_INVALID, "k_new and v_new go together");
    if (!a->append_pos_dev && (a->append_pos < 0 || a->append_pos >= a->L))
      return fail(SAGA_ERR_INVALID, "append_pos outside [0, L)");
    if (a->append_pos_dev && a->shards > 1)
      return fail(SAGA_ERR_UNSUPPORTED, "a device-side append position is not supported with sharding");
  }
  return SAGA_OK;
}

int mode_of(int op) {
  switch (op) {
    case SAGA_OP_ATOPN_DECODE: return saga::MODE_AMORTIZED;
    case SAGA_OP_ATOPN_CALIBRATE: return saga::MODE_CALIBRATE;
    case SAGA_OP_DENSE_DECODE: return saga::MODE_DENSE;
    default: return saga::MODE_LOGITS;
  }
}

int run_attn(const SagaAttnArgs* a, int op, void* stream) {
  g_err.clear();
  g_launched.clear();
  int rc = check_shapes(a);
  if (rc) return rc;
  if (a->B == 0) return SAGA_OK;  // nothing to do; empty tensors may carry NULL pointers
  rc = check_attn(a, op);
  if (rc) return rc;
  std::string err;
  rc = saga::launch_decode(a, mode_of(op), reinterpret_cast<cudaStream_t>(stream), &err, &g_launched);
  if (rc) return fail(rc, err);
  return SAGA_OK;
}

}  // namespace

namespace saga {
// Error reporting for entry points defined in other files.
int abi_fail(int code, const std::string& msg) { return fail(code, msg); }
// The full host-side validation of an attention call (no launch).
int abi_check(const SagaAttnArgs* a, int op) {
  int rc = check_shapes(a);
  if (rc || a->B == 0) return rc;
  return check_attn(a, op);
}
}  // namespace saga

extern "C" {

size_t saga_workspace_bytes(const SagaAttnArgs* args, int32_t op) {
  g_err.clear();
  if (op < SAGA_OP_ATOPN_DECODE || op > SAGA_OP_LOGITS) {
    fail(SAGA_ERR_INVALID, "unknown op");
    return 0;
  }
  if (check_shapes(args)) return 0;
  if (op == SAGA_OP_LOGITS) return 256;
  if (args->B == 0) return 256;
  saga::DecodePlan pl;
  std::string err;
  if (saga::make_decode_plan(args, mode_of(op), &pl, &err)) {
    fail(SAGA_ERR_UNSUPPORTED, err);
    return 0;
  }
  return pl.ws_total;
}

int saga_atopn_decode(const SagaAttnArgs* args, void* stream) {
  return run_attn(args, SAGA_OP_ATOPN_DECODE, stream);
}

int saga_atopn_calibrate(const SagaAttnArgs* args, void* stream) {
  return run_attn(args, SAGA_OP_ATOPN_CALIBRATE, stream);
}

int saga_dense_decode(const SagaAttnArgs* args, void* stream) {
  return run_attn(args, SAGA_OP_DENSE_DECODE, stream);
}

int saga_attn_logits(const SagaAttnArgs* args, void* stream) {
  return run_attn(args, SAGA_OP_LOGITS, stream);
}

int saga_transform_threshold(int32_t dtype, const void* logits, int64_t ld, int32_t rows, int32_t L,
                             const float* thr, int32_t tail, float* t_out, float* m_out, float* s_out,
                             void* stream) {
  g_err.clear();
  g_launched.clear();
  if (!is_fp(dtype)) return fail(SAGA_ERR_INVALID, "dtype must be bf16, fp16 or fp32");
  if (rows < 0 || L <= 0 || ld < L || tail <= 0) return fail(SAGA_ERR_INVALID, "bad rows / L / ld / tail");
  if (rows > 0 && (!logits || !thr || !t_out)) return fail(SAGA_ERR_INVALID, "NULL pointer");
  std::string err;
  int rc = saga::launch_transform(dtype, logits, ld, rows, L, thr, tail, t_out, m_out, s_out,
                                  reinterpret_cast<cudaStream_t>(stream), &err);
  if (rc) return fail(rc, err);
  g_launched = "transform_kernel";
  return SAGA_OK;
}

int saga_threshold_select(int32_t dtype, const void* x, int64_t ldx, int32_t rows, int32_t L, int32_t k,
                          const float* thr, int32_t thr_count, void* vals, int64_t* idx, int32_t* counts,
                          void* stream) {
  g_err.clear();
  g_launched.clear();
  if (!is_fp(dtype)) return fail(SAGA_ERR_INVALID, "dtype must be bf16, fp16 or fp32");
  if (rows < 0 || L <= 0 || ldx < L || k <= 0) return fail(SAGA_ERR_INVALID, "bad rows / L / ldx / k");
  if (thr_count <= 0) return fail(SAGA_ERR_INVALID, "thr_count must be positive");
  if (rows > 0 && (!x || !thr || !vals || !idx)) return fail(SAGA_ERR_INVALID, "NULL pointer");
  std::string err;
  int rc = saga::launch_select(dtype, x, ldx, rows, L, k, thr, thr_count, vals, idx, counts,
                               reinterpret_cast<cudaStream_t>(stream), &err);
  if (rc) return fail(rc, err);
  g_launched = "select_kernel";
  return SAGA_OK;
}

int saga_gather_output(int32_t dtype, const void* w, const int64_t* idx, int32_t K, int32_t input_is_logits,
                       const void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl, int32_t B, int32_t Hq,
                       int32_t Hv, int32_t D, int32_t L, void* out, int64_t o_sb, int64_t o_sh, void* stream) {
  g_err.clear();
  g_launched.clear();
  if (!is_fp(dtype)) return fail(SAGA_ERR_INVALID, "dtype must be bf16, fp16 or fp32");
  if (B < 0 || Hq <= 0 || Hv <= 0 || Hq % Hv || D <= 0 || D % 32 || L <= 0 || K <= 0)
    return fail(SAGA_ERR_INVALID, "bad shapes");
  if (B > 0 && (!w || !idx || !v || !out)) return fail(SAGA_ERR_INVALID, "NULL pointer");
  std::string err;
  int rc = saga::launch_gather(dtype, w, idx, K, input_is_logits, v, v_sb, v_sh, v_sl, B, Hq, Hv, D, L, out,
                               o_sb, o_sh, reinterpret_cast<cudaStream_t>(stream), &err);
  if (rc) return fail(rc, err);
  g_launched = "gather_kernel";
  return SAGA_OK;
}

int saga_ipc_handle(const void* ptr, void* handle64, size_t* offset) {
  g_err.clear();
  if (!ptr || !handle64 || !offset) return fail(SAGA_ERR_INVALID, "NULL argument");
  using GetRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static GetRange get_range = nullptr;
  if (!get_range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(SAGA_ERR_CUDA, "cuMemGetAddressRange unavailable");
    get_range = reinterpret_cast<GetRange>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(SAGA_ERR_INVALID, "pointer is not device memory");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(SAGA_ERR_CUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  memcpy(handle64, &h, sizeof(h));
  *offset = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return SAGA_OK;
}

int saga_ipc_open(const void* handle64, void** ptr) {
  g_err.clear();
  if (!handle64 || !ptr) return fail(SAGA_ERR_INVALID, "NULL handle or pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(SAGA_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  *ptr = p;
  return SAGA_OK;
}

int saga_ipc_close(void* ptr) {
  g_err.clear();
  if (!ptr) return SAGA_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(SAGA_ERR_CUDA, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return SAGA_OK;
}

int saga_kv_append(int32_t dtype, int32_t B, int32_t Hk, int32_t Hv, int32_t D, int32_t L, int32_t pos, void* k,
                   int64_t k_sb, int64_t k_sh, int64_t k_sl, void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl,
                   const void* k_new, int64_t kn_sb, int64_t kn_sh, const void* v_new, int64_t vn_sb,
                   int64_t vn_sh, void* stream) {
  g_err.clear();
  g_launched.clear();
  if (!is_fp(dtype)) return fail(SAGA_ERR_INVALID, "dtype must be bf16, fp16 or fp32");
  if (B < 0 || Hk <= 0 || Hv <= 0 || D <= 0 || L <= 0) return fail(SAGA_ERR_INVALID, "bad shapes");
  if (pos < 0 || pos >= L) return fail(SAGA_ERR_INVALID, "pos outside [0, L)");
  if (B > 0 && (!k || !v || !k_new || !v_new)) return fail(SAGA_ERR_INVALID, "NULL pointer");
  std::string err;
  int rc = saga::launch_append(dtype, B, Hk, Hv, D, pos, k, k_sb, k_sh, k_sl, v, v_sb, v_sh, v_sl, k_new, kn_sb,
                               kn_sh, v_new, vn_sb, vn_sh, reinterpret_cast<cudaStream_t>(stream), &err);
  if (rc) return fail(rc, err);
  g_launched = "append_kernel";
  return SAGA_OK;
}

const char* saga_last_error(void) { return g_err.c_str(); }

const char* saga_version(void) { return "saga_b200 0.1.0 (sm_100a)"; }

const char* saga_last_launches(void) { return g_launched.c_str(); }

}  // extern "C"
