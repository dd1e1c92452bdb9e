// Host launchers of the unfused kernels (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace saga {

int launch_select(int dt, const void* x, int64_t ldx, int rows, int L, int k, const float* thr,
                  int thr_count, void* vals, int64_t* idx, int* counts, cudaStream_t st, std::string* err);

int launch_transform(int dt, const void* x, int64_t ld, int rows, int L, const float* thr, int tail,
                     float* t_out, float* m_out, float* s_out, cudaStream_t st, std::string* err);

int launch_gather(int dt, const void* w, const int64_t* idx, int K, int logits, const void* v, int64_t v_sb,
                  int64_t v_sh, int64_t v_sl, int B, int Hq, int Hv, int D, int L, void* out, int64_t o_sb,
                  int64_t o_sh, cudaStream_t st, std::string* err);

int launch_append(int dt, int B, int Hk, int Hv, int D, int pos, void* k, int64_t k_sb, int64_t k_sh,
                  int64_t k_sl, void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl, const void* kn, int64_t kn_sb,
                  int64_t kn_sh, const void* vn, int64_t vn_sb, int64_t vn_sh, cudaStream_t st,
                  std::string* err);

}  // namespace saga
