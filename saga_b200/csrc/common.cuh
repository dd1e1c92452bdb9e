// Shared device helpers of the saga_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/saga_b200.h"

namespace saga {

constexpr int kThreads = 256;  // 8 warps per CTA in every kernel here
constexpr int kWarps = kThreads / 32;
constexpr int kTile = 128;     // positions per score tile
constexpr int kTail = 256;     // attention.py:136, tail_size of the max estimate
constexpr int kTraceCols = 128;  // int64 stamps per CTA in the optional phase trace
constexpr unsigned long long kWaitLimitNs = 500ull * 1000ull * 1000ull;  // 0.5 s

// ---------------------------------------------------------------------------
// Number formats. `round` replays the reference's rounding of a float result
// to the tensor dtype (round to nearest even); fp32 is the identity.
// ---------------------------------------------------------------------------
template <typename T> struct Num;

template <> struct Num<__nv_bfloat16> {
  static constexpr int kDType = SAGA_BF16;
  static constexpr bool kLowp = true;
  static constexpr int kKeyBits = 16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  // Order-preserving unsigned key of a value already representable in bf16.
  __device__ __forceinline__ static uint32_t key(float x) {
    uint32_t u = __float_as_uint(x) >> 16;
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  }
  __device__ __forceinline__ static float unkey(uint32_t k) {
    uint32_t u = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __uint_as_float(u << 16);
  }
  // Neighbours of a positive finite bf16 value.
  __device__ __forceinline__ static float next_up(float x) { return __uint_as_float(((__float_as_uint(x) >> 16) + 1u) << 16); }
  __device__ __forceinline__ static float next_down(float x) { return __uint_as_float(((__float_as_uint(x) >> 16) - 1u) << 16); }
};

template <> struct Num<__half> {
  static constexpr int kDType = SAGA_FP16;
  static constexpr bool kLowp = true;
  static constexpr int kKeyBits = 16;
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float round(float x) { return __half2float(__float2half_rn(x)); }
  __device__ __forceinline__ static uint32_t key(float x) {
    uint32_t u = __half_as_ushort(__float2half_rn(x));
    return (u & 0x8000u) ? (~u & 0xFFFFu) : (u | 0x8000u);
  }
  __device__ __forceinline__ static float unkey(uint32_t k) {
    uint32_t u = (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
    return __half2float(__ushort_as_half((unsigned short)u));
  }
  // Neighbours of a positive finite fp16 value.
  __device__ __forceinline__ static float next_up(float x) {
    return __half2float(__ushort_as_half((unsigned short)(__half_as_ushort(__float2half_rn(x)) + 1u)));
  }
  __device__ __forceinline__ static float next_down(float x) {
    return __half2float(__ushort_as_half((unsigned short)(__half_as_ushort(__float2half_rn(x)) - 1u)));
  }
};

template <> struct Num<float> {
  static constexpr int kDType = SAGA_FP32;
  static constexpr bool kLowp = false;
  static constexpr int kKeyBits = 32;
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
  __device__ __forceinline__ static float round(float x) { return x; }
  __device__ __forceinline__ static uint32_t key(float x) {
    uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  }
  __device__ __forceinline__ static float unkey(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
  }
  __device__ __forceinline__ static float next_up(float x) { return nextafterf(x, INFINITY); }
  __device__ __forceinline__ static float next_down(float x) { return nextafterf(x, -INFINITY); }
};

// Load 8 consecutive elements (16 B for 16-bit types, 32 B for fp32) as floats.
template <typename T>
__device__ __forceinline__ void load8f(const T* p, float* f);

template <>
__device__ __forceinline__ void load8f<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <>
__device__ __forceinline__ void load8f<__half>(const __half* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <>
__device__ __forceinline__ void load8f<float>(const float* p, float* f) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Load N consecutive elements (N in {2, 4}) as floats, one vector load.
template <typename T, int N>
__device__ __forceinline__ void loadNf(const T* p, float* f) {
  if constexpr (sizeof(T) == 2 && N == 4) {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = Num<T>::to_f(h[i]);
  } else if constexpr (sizeof(T) == 2 && N == 2) {
    uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    const T* h = reinterpret_cast<const T*>(&u);
    f[0] = Num<T>::to_f(h[0]);
    f[1] = Num<T>::to_f(h[1]);
  } else if constexpr (sizeof(T) == 4 && N == 4) {
    float4 a = *reinterpret_cast<const float4*>(p);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  } else {
    float2 a = *reinterpret_cast<const float2*>(p);
    f[0] = a.x; f[1] = a.y;
  }
}

// Additive mask value at an element (bool: 1.0 / 0.0; else the element itself).
template <typename T>
__device__ __forceinline__ float mask_value(const void* m, int mdt, int64_t off) {
  if (mdt == SAGA_BOOL) return reinterpret_cast<const uint8_t*>(m)[off] ? 1.0f : 0.0f;
  return Num<T>::to_f(reinterpret_cast<const T*>(m)[off]);
}

// torch.clamp(min=1e-30) keeps NaN (fmaxf would not).
__device__ __forceinline__ float clamp_min_keep_nan(float x, float lo) { return (x < lo) ? lo : x; }

// ---------------------------------------------------------------------------
// Warp / block reductions with a fixed order (results are run-to-run stable).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Inclusive prefix sum across the warp.
__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

// Reduces v[0..15] with `op` across the 32 lanes of the warp by halving the
// live values at each butterfly step (15 shuffles instead of 16 x 5). Lanes
// 2k and 2k + 1 return the reduction of value k. The combination order is
// fixed, so sums are identical from run to run.
template <typename V, typename Op>
__device__ __forceinline__ V warp_reduce16(const V (&v)[16], Op op) {
  const int lane = threadIdx.x & 31;
  V a[8], b[4], c[2];
  bool up = (lane & 16) != 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const V send = up ? v[k] : v[k + 8];
    a[k] = op(up ? v[k + 8] : v[k], __shfl_xor_sync(0xffffffffu, send, 16));
  }
  up = (lane & 8) != 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const V send = up ? a[k] : a[k + 4];
    b[k] = op(up ? a[k + 4] : a[k], __shfl_xor_sync(0xffffffffu, send, 8));
  }
  up = (lane & 4) != 0;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const V send = up ? b[k] : b[k + 2];
    c[k] = op(up ? b[k + 2] : b[k], __shfl_xor_sync(0xffffffffu, send, 4));
  }
  up = (lane & 2) != 0;
  V d = op(up ? c[1] : c[0], __shfl_xor_sync(0xffffffffu, up ? c[0] : c[1], 2));
  return op(d, __shfl_xor_sync(0xffffffffu, d, 1));
}

// Division by a runtime divisor d >= 1 through a 64-bit reciprocal: exact for
// x * d < 2^32 (q = floor(x * ceil(2^32 / d) / 2^32)).
struct FastDiv {
  uint64_t m;
  __device__ __forceinline__ explicit FastDiv(uint32_t d) : m(((1ull << 32) + d - 1) / d) {}
  __device__ __forceinline__ uint32_t div(uint32_t x) const { return (uint32_t)((x * m) >> 32); }
};

// NaN-propagating max (torch.max semantics): NaN wins.
__device__ __forceinline__ float nanmax(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fffffff) : fmaxf(a, b);
}
__device__ __forceinline__ float warp_nanmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = nanmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Inter-CTA group barrier with a bounded wait. Every thread of the CTA calls
// it. The CTA's prior global writes are published (bar.sync + gpu-scope fence
// by thread 0, then the arrival), and the caller sees the other CTAs' writes
// after it returns. `arrive` = false waits without arriving. On timeout the
// status word gets SAGA_STATUS_WAIT_TIMEOUT and the function returns false
// (the caller carries on; the outputs are then invalid, the GPU is not hung).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool group_barrier(int* ctr, int target, bool arrive, int* status,
                                              int* smem_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (arrive) atomicAdd(ctr, 1);
    int ok = 1;
    if (ld_acquire_gpu(ctr) < target) {
      // poll the counter; read the clock only every 256 polls
      unsigned long long t0 = 0;
      for (uint32_t i = 1; ld_acquire_gpu(ctr) < target; ++i) {
        __nanosleep(32);
        if ((i & 255u) == 0) {
          const unsigned long long now = globaltimer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            ok = 0;
            if (status) atomicOr(status, SAGA_STATUS_WAIT_TIMEOUT);
            break;
          }
        }
      }
    }
    __threadfence();
    *smem_flag = ok;
  }
  __syncthreads();
  return *smem_flag != 0;
}

// The same barrier across devices (sequence sharding): the counter lives in
// one device's memory and every device's CTAs arrive and poll at system scope.
__device__ __forceinline__ bool group_barrier_sys(int* ctr, int target, int* status, int* smem_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    atomicAdd_system(ctr, 1);
    int ok = 1;
    unsigned long long t0 = 0;
    for (uint32_t i = 1; ld_acquire_sys(ctr) < target; ++i) {
      __nanosleep(64);
      if ((i & 255u) == 0) {
        const unsigned long long now = globaltimer_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitLimitNs) {
          ok = 0;
          if (status) atomicOr(status, SAGA_STATUS_WAIT_TIMEOUT);
          break;
        }
      }
    }
    __threadfence_system();
    *smem_flag = ok;
  }
  __syncthreads();
  return *smem_flag != 0;
}

__device__ __forceinline__ void set_status(int* status, int bits) {
  if (status) atomicOr(status, bits);
}

}  // namespace saga
