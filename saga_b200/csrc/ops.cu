// Unfused kernels of the decode path, one per reference helper:
//   threshold select      triton_atopn.py:6-53 / 59-113 (threshold_topk_fast)
//   threshold transform   attention.py:136-149 (_transform_softmax_threshold)
//   buffer gather/output  attention.py:152-170 (_atopn_gather_and_output)
//   KV append             StaticLayer.update's index_copy_ (speedup.py:119-139 cache)
#include <string>

#include "common.cuh"
#include "ops_internal.h"

namespace saga {

// ---------------------------------------------------------------------------
// threshold select: one CTA per row, 256 positions per round, ascending
// compaction with a warp-ballot block scan (deterministic order).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) select_kernel(const T* __restrict__ x, int64_t ldx, int L, int k,
                                                          const float* __restrict__ thr, int thr_count,
                                                          T* __restrict__ vals, int64_t* __restrict__ idx,
                                                          int* __restrict__ counts) {
  __shared__ int wcount[kWarps];
  __shared__ int running_s;
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float t = thr[thr_count == 1 ? 0 : (r % thr_count)];
  const T* xr = x + (int64_t)r * ldx;
  T* vr = vals + (int64_t)r * k;
  int64_t* ir = idx + (int64_t)r * k;
  if (threadIdx.x == 0) running_s = 0;
  __syncthreads();
  int running = 0;
  for (int base = 0; base < L; base += kThreads) {
    const int i = base + threadIdx.x;
    float xv = 0.f;
    bool pass = false;
    if (i < L) {
      xv = Num<T>::to_f(xr[i]);
      pass = xv > t;  // triton_atopn.py:42 (strict, fp32 compare)
    }
    const unsigned bal = __ballot_sync(0xffffffffu, pass);
    if (lane == 0) wcount[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      if (w < warp) before += wcount[w];
      total += wcount[w];
    }
    if (pass) {
      const int o = running + before + __popc(bal & ((1u << lane) - 1u));
      if (o < k) {
        vr[o] = xr[i];
        ir[o] = i;
      }
    }
    running += total;
    __syncthreads();
  }
  // padding of the unused slots (triton_atopn.py:82-84)
  const int kept = running < k ? running : k;
  for (int o = kept + threadIdx.x; o < k; o += kThreads) {
    vr[o] = Num<T>::from_f(-INFINITY);
    ir[o] = 0;
  }
  if (threadIdx.x == 0 && counts) counts[r] = running;
}

// ---------------------------------------------------------------------------
// threshold transform: one CTA per row.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) transform_kernel(const T* __restrict__ x, int64_t ld, int L,
                                                             const float* __restrict__ thr, int tail,
                                                             float* __restrict__ t_out, float* __restrict__ m_out,
                                                             float* __restrict__ s_out) {
  __shared__ float red[kWarps];
  const int r = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T* xr = x + (int64_t)r * ld;
  const int tl = tail < L ? tail : L;
  // m = max of the last tl logits (attention.py:142-143)
  float m = -INFINITY;
  for (int i = L - tl + threadIdx.x; i < L; i += kThreads) m = nanmax(m, Num<T>::to_f(xr[i]));
  m = warp_nanmax(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = red[0];
  for (int w = 1; w < kWarps; ++w) m = nanmax(m, red[w]);
  __syncthreads();
  // s = exp(x - m).sum() with the dtype roundings (attention.py:145)
  float s = 0.f;
  for (int i = threadIdx.x; i < L; i += kThreads)
    s += Num<T>::round(expf(Num<T>::round(__fsub_rn(Num<T>::to_f(xr[i]), m))));
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < kWarps; ++w) tot += red[w];
    tot = Num<T>::round(tot);
    const float th = clamp_min_keep_nan(thr[r], 1e-30f);
    t_out[r] = __fadd_rn(m, logf(__fmul_rn(th, tot)));  // attention.py:147
    if (m_out) m_out[r] = m;
    if (s_out) s_out[r] = tot;
  }
}

// ---------------------------------------------------------------------------
// buffer gather: one CTA per row (b, h); weights -> probabilities, then
// sum_i p_i V[vh, idx_i, :] in fp32.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) gather_kernel(const T* __restrict__ w, const int64_t* __restrict__ idx,
                                                          int K, int logits, const T* __restrict__ v, int64_t v_sb,
                                                          int64_t v_sh, int64_t v_sl, int Hq, int Hv, int D, int L,
                                                          T* __restrict__ out, int64_t o_sb, int64_t o_sh) {
  extern __shared__ float gsm[];  // p[K] then red[kWarps][D]
  __shared__ float redv[kWarps];
  const int r = blockIdx.x;
  const int b = r / Hq, h = r % Hq;
  const int vh = h / (Hq / Hv);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const T* wr = w + (int64_t)r * K;
  const int64_t* ir = idx + (int64_t)r * K;
  float* pbuf = gsm;
  float* red = gsm + K;
  float m = -INFINITY;
  if (logits) {
    for (int i = threadIdx.x; i < K; i += kThreads) m = nanmax(m, Num<T>::to_f(wr[i]));
    m = warp_nanmax(m);
    if (lane == 0) redv[warp] = m;
    __syncthreads();
    m = redv[0];
    for (int q = 1; q < kWarps; ++q) m = nanmax(m, redv[q]);
    __syncthreads();
  }
  float s = 0.f;
  for (int i = threadIdx.x; i < K; i += kThreads) {
    const float x = Num<T>::to_f(wr[i]);
    const float e = logits ? expf(x - m) : x;
    pbuf[i] = e;
    s += e;
  }
  s = warp_sum(s);
  if (lane == 0) redv[warp] = s;
  __syncthreads();
  float tot = 0.f;
  for (int q = 0; q < kWarps; ++q) tot += redv[q];
  // attention.py:158-161: softmax, or p / clamp(sum p, 1e-12) in the dtype
  const float denom = logits ? tot : fmaxf(Num<T>::round(tot), 1e-12f);
  for (int i = threadIdx.x; i < K; i += kThreads) pbuf[i] = pbuf[i] / denom;
  __syncthreads();
  // warps split the buffer, lanes split D
  const T* vb = v + (int64_t)b * v_sb + (int64_t)vh * v_sh;
  for (int d0 = 0; d0 < D; d0 += 32) {
    const int d = d0 + lane;
    float acc = 0.f;
    if (d < D) {
      for (int i = warp; i < K; i += kWarps) {
        const float pi = pbuf[i];
        if (pi != 0.f) {
          int64_t pos = ir[i];
          pos = pos < 0 ? 0 : (pos >= L ? L - 1 : pos);
          acc = fmaf(pi, Num<T>::to_f(vb[pos * v_sl + d]), acc);
        }
      }
    }
    red[warp * D + (d < D ? d : 0)] = (d < D) ? acc : 0.f;
    __syncthreads();
    if (warp == 0 && d < D) {
      float o = 0.f;
      for (int q = 0; q < kWarps; ++q) o += red[q * D + d];
      out[(int64_t)b * o_sb + (int64_t)h * o_sh + d] = Num<T>::from_f(o);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// KV append: grid (B, Hk + Hv), one row of D elements per CTA.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void append_kernel(int Hk, int D, int pos, T* k, int64_t k_sb, int64_t k_sh, int64_t k_sl, T* v,
                              int64_t v_sb, int64_t v_sh, int64_t v_sl, const T* kn, int64_t kn_sb, int64_t kn_sh,
                              const T* vn, int64_t vn_sb, int64_t vn_sh) {
  const int b = blockIdx.x, hh = blockIdx.y;
  if (hh < Hk) {
    T* dst = k + (int64_t)b * k_sb + (int64_t)hh * k_sh + (int64_t)pos * k_sl;
    const T* src = kn + (int64_t)b * kn_sb + (int64_t)hh * kn_sh;
    for (int d = threadIdx.x; d < D; d += blockDim.x) dst[d] = src[d];
  } else {
    const int vh = hh - Hk;
    T* dst = v + (int64_t)b * v_sb + (int64_t)vh * v_sh + (int64_t)pos * v_sl;
    const T* src = vn + (int64_t)b * vn_sb + (int64_t)vh * vn_sh;
    for (int d = threadIdx.x; d < D; d += blockDim.x) dst[d] = src[d];
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
#define SAGA_DISPATCH(dt, ...)                                   \
  do {                                                           \
    if ((dt) == SAGA_BF16) {                                     \
      using T = __nv_bfloat16;                                   \
      __VA_ARGS__;                                               \
    } else if ((dt) == SAGA_FP16) {                              \
      using T = __half;                                          \
      __VA_ARGS__;                                               \
    } else {                                                     \
      using T = float;                                           \
      __VA_ARGS__;                                               \
    }                                                            \
  } while (0)

static int check_launch(std::string* err, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *err = std::string(what) + ": " + cudaGetErrorString(e);
    return SAGA_ERR_CUDA;
  }
  return SAGA_OK;
}

int launch_select(int dt, const void* x, int64_t ldx, int rows, int L, int k, const float* thr,
                  int thr_count, void* vals, int64_t* idx, int* counts, cudaStream_t st, std::string* err) {
  if (rows == 0) return SAGA_OK;
  SAGA_DISPATCH(dt, select_kernel<T><<<rows, kThreads, 0, st>>>(
                        reinterpret_cast<const T*>(x), ldx, L, k, thr, thr_count,
                        reinterpret_cast<T*>(vals), idx, counts));
  return check_launch(err, "select_kernel");
}

int launch_transform(int dt, const void* x, int64_t ld, int rows, int L, const float* thr, int tail,
                     float* t_out, float* m_out, float* s_out, cudaStream_t st, std::string* err) {
  if (rows == 0) return SAGA_OK;
  SAGA_DISPATCH(dt, transform_kernel<T><<<rows, kThreads, 0, st>>>(reinterpret_cast<const T*>(x), ld, L, thr,
                                                                   tail, t_out, m_out, s_out));
  return check_launch(err, "transform_kernel");
}

int launch_gather(int dt, const void* w, const int64_t* idx, int K, int logits, const void* v, int64_t v_sb,
                  int64_t v_sh, int64_t v_sl, int B, int Hq, int Hv, int D, int L, void* out, int64_t o_sb,
                  int64_t o_sh, cudaStream_t st, std::string* err) {
  const int rows = B * Hq;
  if (rows == 0) return SAGA_OK;
  const size_t smem = (size_t)(K + kWarps * D) * sizeof(float);
  if (smem > 200 * 1024) {
    *err = "gather buffer too large";
    return SAGA_ERR_UNSUPPORTED;
  }
  SAGA_DISPATCH(dt, {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(gather_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    gather_kernel<T><<<rows, kThreads, smem, st>>>(reinterpret_cast<const T*>(w), idx, K, logits,
                                                   reinterpret_cast<const T*>(v), v_sb, v_sh, v_sl, Hq, Hv, D, L,
                                                   reinterpret_cast<T*>(out), o_sb, o_sh);
  });
  return check_launch(err, "gather_kernel");
}

int launch_append(int dt, int B, int Hk, int Hv, int D, int pos, void* k, int64_t k_sb, int64_t k_sh,
                  int64_t k_sl, void* v, int64_t v_sb, int64_t v_sh, int64_t v_sl, const void* kn, int64_t kn_sb,
                  int64_t kn_sh, const void* vn, int64_t vn_sb, int64_t vn_sh, cudaStream_t st,
                  std::string* err) {
  if (B == 0) return SAGA_OK;
  SAGA_DISPATCH(dt, append_kernel<T><<<dim3(B, Hk + Hv), 128, 0, st>>>(
                        Hk, D, pos, reinterpret_cast<T*>(k), k_sb, k_sh, k_sl, reinterpret_cast<T*>(v), v_sb,
                        v_sh, v_sl, reinterpret_cast<const T*>(kn), kn_sb, kn_sh,
                        reinterpret_cast<const T*>(vn), vn_sb, vn_sh));
  return check_launch(err, "append_kernel");
}

}  // namespace saga
