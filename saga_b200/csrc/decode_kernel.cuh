// Fused SAGA decode attention on sm_100a: one persistent kernel per step.
//
// Work item = (group g = batch x key head, chunk j of the sequence). The C
// chunks of a group run concurrently (cooperative launch, static round-robin
// assignment). Per item:
//   score   the G query heads of the group against the chunk's keys. For
//           bf16/fp16 with G <= 16: TMA streams 128-position K tiles (128-B
//           swizzle) through a ring of shared-memory stages; one thread issues
//           tcgen05 UMMAs (M = 128 positions, N = 16 query-head slots, K = D)
//           into a double-buffered TMEM accumulator; four warps read it back
//           (tcgen05.ld) and finalise head pairs with packed conversions;
//           two more warps fold each stored tile into the per-head exp-sum /
//           maximum while the next tiles stream. Otherwise CUDA-core FMAs.
//           Either way the reference rounding chain is applied (GEMM -> dtype,
//           * scaling -> dtype, + mask -> dtype; attention.py:113-128) and the
//           logits stay in shared memory, position-major ([pos][head slot]);
//   then, by mode:
//   amortized (attention.py:192-209): every CTA scores the last 256 positions
//           itself, so the tail max m (attention.py:142-143) needs no exchange,
//           and the exp-sum of its chunk (145) accumulates during scoring; one
//           exchange of the partial sums gives the logit threshold (147);
//           strict selection (triton_atopn.py:42); one exchange of per-chunk
//           counts keeps the K = min(2N, L) lowest passing positions; softmax
//           weights exp(l - stabiliser);
//   calibrate (attention.py:173-189): global max and sum of exp, exact N-th
//           largest logit by an 8-bit-per-pass radix select over the group,
//           its probability as the threshold, top-N set (ties by position),
//           weights = the dtype-rounded probabilities;
//   dense   (attention.py:64-85): weights exp(l - m_chunk) for all positions;
//   then the V gather (every needed value row fetched once per value head),
//   a partial (m, l, o[D]) per head, and a merge split across the chunks.
//
// Exchanges between the chunks of a group go through epoch-tagged 64-bit
// slots (32-bit launch tag | 32-bit value): a reader polls the data itself,
// one L2 round trip when it is ready, with no separate counter. The group's
// last chunk to finish advances the epoch for the next launch.
#pragma once

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "common.cuh"
#include "decode_internal.h"
#include "tc.cuh"

namespace saga {

// ---------------------------------------------------------------------------
// per-CTA shared scalars
// ---------------------------------------------------------------------------
struct Misc {
  uint64_t full[kMaxStages];   // K tile landed (TMA complete_tx)
  uint64_t empty[kMaxStages];  // K stage free again (UMMA commit)
  uint64_t tfull[2];           // TMEM accumulator ready (UMMA commit)
  uint64_t tempty[2];          // TMEM accumulator drained (4 epilogue warps)
  uint32_t tmem_slot;
  int abort;
  uint32_t tag;                // exchange tag of this launch for the current group
  int stored;                  // tiles x 4 epilogue warps stored to SMEM (this item)
  uint32_t tkey[kMaxG];        // order-preserving keys of the tail max (fp32 path)
  float ered[2][kMaxG];        // per-helper-warp partial exp-sums
  float emax[2][kMaxG];        // per-helper-warp partial maxima
  float esum4[4][16];          // per-epilogue-warp partial exp-sums (first head pairs)
  float emax4[4][16];          // per-epilogue-warp partial maxima (first head pairs)
  int mready;                  // tail max published (this item)
  int tcount;                  // epilogue warps done with the tail tiles (this item)
  float tmax4[4][16];          // per-epilogue-warp tail maxima
  int cntw[8][kMaxG];          // per-warp selection counts
  float m[kMaxG];      // tail max / global max
  float t[kMaxG];      // logit threshold / N-th logit
  float s[kMaxG];      // exp-sum
  float aux[kMaxG];    // stabiliser of the weights / p_N
  int i0[kMaxG];       // prefix / want
  int i1[kMaxG];       // keep / key prefix
  int i2[kMaxG];
  int i3[kMaxG];
  float lsum[kMaxG];
  int gstart[kMaxGatherGroups + 1];  // gather groups: list ranges
  int gvh[kMaxGatherGroups];
  int ghb[kMaxGatherGroups];
  int ngroups;
  int flag;
  int last;
};
static_assert(sizeof(Misc) <= 6144, "Misc must fit its 6 KB slot");

// Per-thread pipeline positions kept across items (only role threads use theirs).
struct Ring {
  uint32_t ps = 0, pph = 0;   // producer stage / phase
  uint32_t ms = 0, mph = 0;   // UMMA issuer stage / phase
  uint32_t mb = 0, mbph = 0;  // UMMA issuer TMEM buffer / phase
  uint32_t eb = 0, ebph = 0;  // epilogue TMEM buffer / phase
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Order-preserving unsigned key of any float (NaN with a positive sign bit
// sorts above +inf, so a max over keys propagates it as torch.max does).
__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float funkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// ---------------------------------------------------------------------------
// Packed pairs of 16-bit values
// ---------------------------------------------------------------------------
template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using P = __nv_bfloat162;
  __device__ __forceinline__ static P pack_rn(float a, float b) { return __floats2bfloat162_rn(a, b); }
  __device__ __forceinline__ static float2 unpack(P x) { return __bfloat1622float2(x); }
  __device__ __forceinline__ static P sub(P a, P b) { return __hsub2(a, b); }
};
template <> struct Pair<__half> {
  using P = __half2;
  __device__ __forceinline__ static P pack_rn(float a, float b) { return __floats2half2_rn(a, b); }
  __device__ __forceinline__ static float2 unpack(P x) { return __half22float2(x); }
  __device__ __forceinline__ static P sub(P a, P b) { return __hsub2(a, b); }
};

// ---------------------------------------------------------------------------
// Epoch-tagged exchange slots
// ---------------------------------------------------------------------------
__device__ __forceinline__ void slot_put(unsigned long long* p, uint32_t tag, uint32_t bits) {
  const unsigned long long v = ((unsigned long long)tag << 32) | bits;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long slot_ld(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Wait until the slot carries `tag`; returns its 32-bit value (bounded wait).
__device__ __forceinline__ uint32_t slot_wait(const unsigned long long* p, unsigned long long v, uint32_t tag,
                                              int* status) {
  if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
  unsigned long long t0 = 0;
  for (uint32_t i = 1;; ++i) {
    __nanosleep(32);
    v = slot_ld(p);
    if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
    if ((i & 255u) == 0) {
      const unsigned long long now = globaltimer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        if (status) atomicOr(status, SAGA_STATUS_WAIT_TIMEOUT);
        return (uint32_t)v;
      }
    }
  }
}
// All threads: fetch `count` slots (addresses from `addr(i)`) into dst[i],
// issuing 8 independent loads per thread before waiting on any of them.
template <typename AddrFn>
__device__ __forceinline__ void slots_gather(int count, AddrFn addr, uint32_t tag, uint32_t* dst, int* status) {
  for (int base = threadIdx.x; base < count; base += kThreads * 8) {
    unsigned long long v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + k * kThreads;
      v[k] = (i < count) ? slot_ld(addr(i)) : 0ull;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + k * kThreads;
      if (i < count) dst[i] = slot_wait(addr(i), v[k], tag, status);
    }
  }
}

// The reference's rounding chain for one logit (attention.py:121-126).
template <typename T, bool MASK>
__device__ __forceinline__ float finalize_logit(const DecodeParams& p, float acc, int b, int h, int pos) {
  float l = Num<T>::round(acc);
  l = Num<T>::round(__fmul_rn(l, p.scaling));
  if constexpr (MASK) {
    const int64_t mo = (int64_t)b * p.m_sb + (int64_t)h * p.m_sh + (int64_t)pos * p.m_sl;
    l = Num<T>::round(__fadd_rn(l, mask_value<T>(p.mask, p.mask_dtype, mo)));
  }
  return l;
}

// One term of the reference's exp-sum: exp(l - m) with both steps rounded to
// the dtype (attention.py:145). The fast exp differs from an accurate one by a
// few fp32 ulps, which the rounding to bf16/fp16 absorbs except at rounding
// boundaries; fp32 uses the accurate expf.
template <typename T>
__device__ __forceinline__ float exp_term(float l, float m) {
  const float d = Num<T>::round(__fsub_rn(l, m));
  return Num<T>::round(Num<T>::kLowp ? __expf(d) : expf(d));
}

// ---------------------------------------------------------------------------
// Scoring on CUDA cores (fp32 path, or more than 16 query heads per key head).
// 64-position sub-tiles of K are staged in SMEM with cp.async (rows padded by
// 16 B); thread t scores position t % 64 for the heads of slice t / 64.
// Positions [a, a + cnt) are scored; with max_only they only raise
// misc->tkey (the tail max), else they are stored at sc[(pos - p0) * SH + hl].
// ---------------------------------------------------------------------------
template <typename T, int D, bool MASK>
__device__ void score_range_simt(const DecodeParams& p, int b, int kh, int a, int cnt, int p0, bool max_only,
                                 const float* __restrict__ qf, T* __restrict__ sc, uint8_t* __restrict__ stage,
                                 Misc* misc) {
  constexpr int SUB = 64;
  constexpr int ROWB = D * (int)sizeof(T);
  constexpr int PITCH = ROWB + 16;
  constexpr int CPR = ROWB / 16;
  const int SH = p.sh;
  const T* kbase = reinterpret_cast<const T*>(p.k) + (int64_t)b * p.k_sb + (int64_t)kh * p.k_sh;
  const int nsub = (cnt + SUB - 1) / SUB;
  const int h0 = kh * p.G;

  auto issue = [&](int s) {
    uint8_t* buf = stage + (s & 1) * SUB * PITCH;
    for (int c = threadIdx.x; c < SUB * CPR; c += kThreads) {
      const int r = c / CPR, cc = c % CPR;
      const bool ok = (s * SUB + r) < cnt;
      const T* src = kbase + (int64_t)(ok ? (a + s * SUB + r) : a) * p.k_sl + cc * (16 / (int)sizeof(T));
      cp_async16(buf + r * PITCH + cc * 16, src, ok);
    }
    cp_async_commit();
  };

  const int pos_l = threadIdx.x % SUB;
  const int slice = threadIdx.x / SUB;
  const int hps = (p.G + 3) / 4;
  const int hbeg = slice * hps;
  const int hend = min(p.G, hbeg + hps);

  issue(0);
  for (int s = 0; s < nsub; ++s) {
    if (s + 1 < nsub) {
      issue(s + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const T* krow = reinterpret_cast<const T*>(stage + (s & 1) * SUB * PITCH + pos_l * PITCH);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll 2
    for (int d = 0; d < D; d += 8) {
      float kf[8];
      load8f<T>(krow + d, kf);
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) {
        if (hbeg + hh < hend) {
          const float* qr = qf + (hbeg + hh) * D + d;
          const float4 qa = *reinterpret_cast<const float4*>(qr);
          const float4 qb = *reinterpret_cast<const float4*>(qr + 4);
          float x = acc[hh];
          x = fmaf(kf[0], qa.x, x); x = fmaf(kf[1], qa.y, x);
          x = fmaf(kf[2], qa.z, x); x = fmaf(kf[3], qa.w, x);
          x = fmaf(kf[4], qb.x, x); x = fmaf(kf[5], qb.y, x);
          x = fmaf(kf[6], qb.z, x); x = fmaf(kf[7], qb.w, x);
          acc[hh] = x;
        }
      }
    }
    const int pr = s * SUB + pos_l;
    if (pr < cnt) {
      const int pos = a + pr;
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) {
        const int hl = hbeg + hh;
        if (hl < hend) {
          const float l = finalize_logit<T, MASK>(p, acc[hh], b, h0 + hl, pos);
          if (max_only) atomicMax(&misc->tkey[hl], fkey(l));
          else sc[(pos - p0) * SH + hl] = Num<T>::from_f(l);
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Scoring on the tensor cores (bf16 / fp16, G <= 16).
//   warp 0 lane 0: TMA producer of 128 x D key tiles (ring of ns stages);
//   warp 1 lane 0: UMMA issuer, D(128 x 16, fp32 in TMEM) = K_tile . Q^T;
//   warps 4-7    : epilogue, lane = position, 16 columns = query-head slots,
//                  finalised in pairs, 32 B stored per position;
//   warps 2-3    : helpers, per-head exp-sum (amortized) and maximum of each
//                  stored tile, overlapped with the next tiles.
// The tile sequence is n_pre tail tiles (global tile indices pre0 ...), stored
// to the tail scratch, then the chunk's own tiles. The query operand (16 rows,
// zero padded beyond G) is written into SMEM in the same 128-B swizzled
// K-major layout the TMA produces for the key tiles.
// ---------------------------------------------------------------------------
template <typename T, int D, int MODE, bool MASK>
__device__ void score_chunk_tc(const DecodeParams& p, int b, int kh, int p0, int n, int pre0, int n_pre,
                               T* __restrict__ sc, T* __restrict__ tsc, uint8_t* __restrict__ qop,
                               uint8_t* __restrict__ ring, Misc* misc, Ring& rg, uint32_t tmem_base) {
  using PT = Pair<T>;
  using P2 = typename PT::P;
  constexpr int KB = D / 64;  // 128-byte K blocks per row
  constexpr uint32_t TILE_BYTES = 128u * D * 2u;
  constexpr uint32_t IDESC = umma_idesc_f16(Num<T>::kDType == SAGA_BF16 ? 1u : 0u, 128, 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.G, NS = p.ns;
  const int h0 = kh * G;
  const int ntl = (n + 127) / 128;
  const int nseq = n_pre + ntl;
  const int tail_start = p.L - p.tail;

  // B operand: query heads of the group as 16 rows x D, swizzled.
  for (int i = threadIdx.x; i < 16 * (D / 8); i += kThreads) {
    const int h = i / (D / 8), c8 = i % (D / 8);
    const int kb = c8 >> 3, c = c8 & 7;
    alignas(16) T vals[8];
    const T* src = reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)(h0 + h) * p.q_sh + c8 * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) vals[e] = (h < G) ? src[e] : Num<T>::from_f(0.f);
    *reinterpret_cast<uint4*>(qop + kb * 2048 + h * 128 + ((c ^ (h & 7)) << 4)) = *reinterpret_cast<uint4*>(vals);
  }
  if (threadIdx.x == 0) {
    misc->stored = 0;
    misc->mready = 0;
    misc->tcount = 0;
  }
  fence_proxy_async_smem();
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int q = 0; q < nseq && !misc->abort; ++q) {
        if (!mbar_wait(&misc->empty[rg.ps], rg.pph ^ 1u, p.status)) {
          misc->abort = 1;
          break;
        }
        const int y = (q < n_pre) ? (pre0 + q) * 128 : p0 + (q - n_pre) * 128;
        mbar_arrive_expect_tx(&misc->full[rg.ps], TILE_BYTES);
        uint8_t* dst = ring + rg.ps * TILE_BYTES;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          tma_load_4d(dst + kb * 16384, &p.tmap, kb * 64, y, kh, b, &misc->full[rg.ps]);
        ++issued;
        if (p.trace && blockIdx.x < 1024 && q < 16) p.trace[blockIdx.x * 64 + 16 + q] = clock64();
        if (++rg.ps == (uint32_t)NS) {
          rg.ps = 0;
          rg.pph ^= 1u;
        }
      }
      if (misc->abort) {
        // drain: the last issued tiles may still be landing
        uint32_t s = rg.ps, ph = rg.pph;
        for (int k = 0; k < min(issued, NS); ++k) {
          if (s == 0) {
            s = NS - 1;
            ph ^= 1u;
          } else {
            --s;
          }
          mbar_wait(&misc->full[s], ph, p.status);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int issued = 0;
      uint32_t last_b = 0, last_ph = 0;
      for (int q = 0; q < nseq && !misc->abort; ++q) {
        if (!mbar_wait(&misc->full[rg.ms], rg.mph, p.status) ||
            !mbar_wait(&misc->tempty[rg.mb], rg.mbph ^ 1u, p.status)) {
          misc->abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(ring + rg.ms * TILE_BYTES);
        const uint32_t b0 = smem_addr(qop);
        const uint32_t dt = tmem_base + rg.mb * 16u;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(dt, umma_desc_sw128(a0 + kb * 16384 + kk * 32), umma_desc_sw128(b0 + kb * 2048 + kk * 32),
                     IDESC, (kb | kk) != 0);
        umma_commit(&misc->empty[rg.ms]);
        umma_commit(&misc->tfull[rg.mb]);
        last_b = rg.mb;
        last_ph = rg.mbph;
        ++issued;
        if (p.trace && blockIdx.x < 1024 && q < 16) p.trace[blockIdx.x * 64 + 32 + q] = clock64();
        if (++rg.ms == (uint32_t)NS) {
          rg.ms = 0;
          rg.mph ^= 1u;
        }
        if (++rg.mb == 2u) {
          rg.mb = 0;
          rg.mbph ^= 1u;
        }
      }
      // all UMMAs of this item complete before their operands are reused
      if (issued) mbar_wait(&misc->tfull[last_b], last_ph, p.status);
    }
  } else if (warp >= 4) {
    // epilogue: TMEM -> logits (reference rounding chain) -> SMEM, 32 B per
    // position; for amortized it also folds the first EJ head pairs of its own
    // tiles into per-head exp-sums and maxima (the helpers take the rest)
    const int q4 = warp - 4;  // TMEM lane quarter of this warp
    const float scl = p.scaling;
    const int EJ = (MODE == MODE_AMORTIZED) ? ((G + 1) / 2) / 2 : 0;
    float es[16], em[16], tm[16];
    P2 m2[8];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      es[k] = 0.f;
      em[k] = -INFINITY;
      tm[k] = -INFINITY;
    }
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) m2[jj] = PT::pack_rn(0.f, 0.f);
    for (int q = 0; q < nseq; ++q) {
      bool ok = mbar_wait(&misc->tfull[rg.eb], rg.ebph, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) misc->abort = 1;
        break;
      }
      tc_fence_after();
      uint32_t r[16];
      tmem_ld16(tmem_base + ((uint32_t)(q4 * 32) << 16) + rg.eb * 16u, r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->tempty[rg.eb]);
      if (++rg.eb == 2u) {
        rg.eb = 0;
        rg.ebph ^= 1u;
      }
      const bool pre = q < n_pre;
      const int pl = pre ? (q * 128 + q4 * 32 + lane) : ((q - n_pre) * 128 + q4 * 32 + lane);
      const int pos = pre ? (pre0 * 128 + pl) : (p0 + pl);
      if (pre || pl < n) {
        alignas(16) P2 outv[8];
        if constexpr (!MASK) {
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            // bmm output in the dtype, * scaling in fp32, rounded again
            const float2 f = PT::unpack(PT::pack_rn(__uint_as_float(r[2 * jj]), __uint_as_float(r[2 * jj + 1])));
            outv[jj] = PT::pack_rn(__fmul_rn(f.x, scl), __fmul_rn(f.y, scl));
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int ha = min(2 * jj, G - 1), hb2 = min(2 * jj + 1, G - 1);
            outv[jj] = PT::pack_rn(finalize_logit<T, true>(p, __uint_as_float(r[2 * jj]), b, h0 + ha, pos),
                                   finalize_logit<T, true>(p, __uint_as_float(r[2 * jj + 1]), b, h0 + hb2, pos));
          }
        }
        if (pre) {
          // tail tile: this position's logits raise the running tail max
          if (pos >= tail_start && pos < p.L) {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
              const float2 f = PT::unpack(outv[jj]);
              tm[2 * jj] = nanmax(tm[2 * jj], f.x);
              tm[2 * jj + 1] = nanmax(tm[2 * jj + 1], f.y);
            }
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(sc + (size_t)pl * 16);
          dst[0] = *reinterpret_cast<const uint4*>(&outv[0]);
          dst[1] = *reinterpret_cast<const uint4*>(&outv[4]);
        }
        if (MODE == MODE_AMORTIZED && !pre) {
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            if (jj < EJ) {
              const float2 f = PT::unpack(outv[jj]);
              em[2 * jj] = fmaxf(em[2 * jj], f.x);
              em[2 * jj + 1] = fmaxf(em[2 * jj + 1], f.y);
              // exp(round(l - m)) rounded, per head (attention.py:145)
              const float2 dd = PT::unpack(PT::sub(outv[jj], m2[jj]));
              const float2 e = PT::unpack(PT::pack_rn(__expf(dd.x), __expf(dd.y)));
              es[2 * jj] += e.x;
              es[2 * jj + 1] += e.y;
            }
          }
        }
      }
      __syncwarp();
      if (!pre && p.trace && blockIdx.x < 1024 && q - n_pre < 16 && q4 == 0 && lane == 0)
        p.trace[blockIdx.x * 64 + 48 + (q - n_pre)] = clock64();
      if (!pre && lane == 0) {
        __threadfence_block();
        atomicAdd(&misc->stored, 1);
      }
      if (pre && q == n_pre - 1) {
        // tail max of the group: warp max, then the last of the four epilogue
        // warps combines and publishes it (helpers and epilogue both wait)
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float v = warp_nanmax(tm[k]);
          if (lane == 0) misc->tmax4[q4][k] = v;
        }
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          if (atomicAdd(&misc->tcount, 1) == 3) {
            __threadfence_block();
            for (int k = 0; k < 16; ++k) {
              const volatile float* t4 = &misc->tmax4[0][0];
              misc->m[k] = nanmax(nanmax(t4[k], t4[16 + k]), nanmax(t4[32 + k], t4[48 + k]));
            }
            __threadfence_block();
            atomicExch(&misc->mready, 1);
          }
        }
        unsigned long long t0 = 0;
        for (uint32_t it = 1; *reinterpret_cast<volatile int*>(&misc->mready) == 0; ++it) {
          __nanosleep(32);
          if (misc->abort) break;
          if ((it & 255u) == 0) {
            const unsigned long long now = globaltimer_ns();
            if (t0 == 0) {
              t0 = now;
            } else if (now - t0 > kWaitLimitNs) {
              set_status(p.status, SAGA_STATUS_WAIT_TIMEOUT);
              break;
            }
          }
        }
        __threadfence_block();
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          if (jj < EJ) m2[jj] = PT::pack_rn(misc->m[2 * jj], misc->m[2 * jj + 1]);
      }
    }
    if (MODE == MODE_AMORTIZED) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        if (k < 2 * EJ) {
          const float sv = warp_sum(es[k]);
          const float mv = warp_max(em[k]);
          if (lane == 0) {
            misc->esum4[q4][k] = sv;
            misc->emax4[q4][k] = mv;
          }
        }
      }
    }
  } else if (warp == 2 || warp == 3) {
    // helpers: tail max first (each helper warp over all tail positions), then
    // the per-head exp-sum and maximum of every stored own tile
    const int hw = warp - 2;
    float m[16], s[16], mx[16];
#pragma unroll
    for (int hl = 0; hl < 16; ++hl) {
      m[hl] = -INFINITY;
      s[hl] = 0.f;
      mx[hl] = -INFINITY;
    }
    auto wait_stored = [&](int target) {
      if (*reinterpret_cast<volatile int*>(&misc->stored) >= target) return true;
      unsigned long long t0 = 0;
      for (uint32_t it = 1; *reinterpret_cast<volatile int*>(&misc->stored) < target; ++it) {
        __nanosleep(64);
        if (misc->abort) return false;
        if ((it & 255u) == 0) {
          const unsigned long long now = globaltimer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            set_status(p.status, SAGA_STATUS_WAIT_TIMEOUT);
            return false;
          }
        }
      }
      return true;
    };
    bool live = true;
    if (n_pre > 0) {
      // the epilogue publishes the tail max once the tail tiles are scored
      unsigned long long t0 = 0;
      for (uint32_t it = 1; *reinterpret_cast<volatile int*>(&misc->mready) == 0; ++it) {
        __nanosleep(64);
        if (misc->abort) {
          live = false;
          break;
        }
        if ((it & 255u) == 0) {
          const unsigned long long now = globaltimer_ns();
          if (t0 == 0) {
            t0 = now;
          } else if (now - t0 > kWaitLimitNs) {
            set_status(p.status, SAGA_STATUS_WAIT_TIMEOUT);
            live = false;
            break;
          }
        }
      }
      __threadfence_block();
#pragma unroll
      for (int hl = 0; hl < 16; ++hl) m[hl] = misc->m[hl];
    }
    const int EJ = (MODE == MODE_AMORTIZED) ? ((G + 1) / 2) / 2 : 0;
    P2 m2[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) m2[jj] = PT::pack_rn(m[2 * jj], m[2 * jj + 1]);
    for (int q = 0; q < ntl && live; ++q) {
      live = wait_stored(4 * (q + 1));
      if (!live) break;
      __threadfence_block();
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int pl = q * 128 + k * 64 + hw * 32 + lane;
        if (pl < n) {
          const uint4* src = reinterpret_cast<const uint4*>(sc + (size_t)pl * 16);
          const uint4 u0 = src[0], u1 = src[1];
          const P2* pp0 = reinterpret_cast<const P2*>(&u0);
          const P2* pp1 = reinterpret_cast<const P2*>(&u1);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            if (2 * jj < G && jj >= EJ) {
              const P2 l2 = jj < 4 ? pp0[jj] : pp1[jj - 4];
              const float2 f = PT::unpack(l2);
              mx[2 * jj] = fmaxf(mx[2 * jj], f.x);
              mx[2 * jj + 1] = fmaxf(mx[2 * jj + 1], f.y);
              if constexpr (MODE == MODE_AMORTIZED) {
                // exp(round(l - m)) rounded, per head (attention.py:145)
                const float2 d = PT::unpack(PT::sub(l2, m2[jj]));
                const float2 e = PT::unpack(PT::pack_rn(__expf(d.x), __expf(d.y)));
                s[2 * jj] += e.x;
                s[2 * jj + 1] += e.y;
              }
            }
          }
        }
      }
    }
#pragma unroll
    for (int hl = 0; hl < 16; ++hl) {
      if (hl < G) {
        const float sv = warp_sum(s[hl]);
        const float mv = warp_max(mx[hl]);
        if (lane == 0) {
          misc->ered[hw][hl] = sv;
          misc->emax[hw][hl] = mv;
        }
      }
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Bit-mask helpers over SMEM words (positions of one head within the chunk).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t keep_lowest_bits(uint32_t w, int r) {
  uint32_t outm = 0;
  for (int i = 0; i < r && w; ++i) {
    const uint32_t lo = w & (0u - w);
    outm |= lo;
    w ^= lo;
  }
  return outm;
}

// Warp-wide: trim bits[0..nw) to their first `keep` set bits (ascending).
__device__ __forceinline__ void warp_trim_bits(uint32_t* bits, int nw, int keep) {
  const int lane = threadIdx.x & 31;
  int running = 0;
  for (int w0 = 0; w0 < nw; w0 += 32) {
    const int w = w0 + lane;
    const uint32_t v = (w < nw) ? bits[w] : 0u;
    const int c = __popc(v);
    const int incl = warp_incl_scan(c);
    const int before = running + incl - c;
    uint32_t nv = v;
    if (before >= keep) nv = 0u;
    else if (before + c > keep) nv = keep_lowest_bits(v, keep - before);
    if (w < nw) bits[w] = nv;
    running += __shfl_sync(0xffffffffu, incl, 31);
  }
  __syncwarp();
}

// Warp-wide: write the set positions of bits (ascending) to dst[0 .. limit).
__device__ __forceinline__ void warp_write_positions(const uint32_t* bits, int nw, int p0, int* dst, int limit) {
  const int lane = threadIdx.x & 31;
  int running = 0;
  for (int w0 = 0; w0 < nw; w0 += 32) {
    const int w = w0 + lane;
    uint32_t v = (w < nw) ? bits[w] : 0u;
    const int c = __popc(v);
    const int incl = warp_incl_scan(c);
    int o = running + incl - c;
    while (v) {
      const int bit = __ffs(v) - 1;
      v &= v - 1;
      if (o < limit) dst[o] = p0 + w * 32 + bit;
      ++o;
    }
    running += __shfl_sync(0xffffffffu, incl, 31);
  }
}

__device__ __forceinline__ bool bit_of(const uint32_t* bits, int i) { return (bits[i >> 5] >> (i & 31)) & 1u; }

// Weight of (local head hl, chunk position i) by mode: exp(l - stabiliser),
// or for calibration the probability rounded to the dtype.
template <typename T, int MODE>
__device__ __forceinline__ float weight_of(const T* sc, int SH, const Misc* misc, int hl, int i) {
  const float l = Num<T>::to_f(sc[i * SH + hl]);
  if constexpr (MODE == MODE_CALIBRATE)
    return Num<T>::round(__fdiv_rn(expf(__fsub_rn(l, misc->m[hl])), misc->s[hl]));
  else
    return __expf(l - misc->aux[hl]);
}

// Slot address: group g, chunk c, local head hl, field k.
__device__ __forceinline__ unsigned long long* slot_at(const DecodeParams& p, int g, int c, int hl, int k) {
  return p.slots + (((size_t)g * p.C + c) * p.G + hl) * (size_t)(p.D + 4) + k;
}
constexpr int kSlotS = 0, kSlotCnt = 1, kSlotM = 2, kSlotL = 3, kSlotO = 4;

// ---------------------------------------------------------------------------
// V gather of one item, in two halves so that the value rows can be in flight
// while the chunks exchange their counts.
//   gather_begin: gather groups = (value head, batch of <= 8 of its query
//     heads); for each group the positions any of its heads selected (bits of
//     hmask[pos]), ascending, form a list (entry = position | head mask << 16 |
//     group << 24). If all rows fit one batch their cp.async copies are issued.
//   gather_end: weights per (entry, head) from the current hmask (a capped
//     chunk may have cleared bits since), wait for the rows, fp32 accumulation
//     per warp, fixed-order reduction across warps, partial (m, l, o[D]) of
//     every head published through the group's tagged slots.
// ---------------------------------------------------------------------------
template <typename T, int D>
__device__ __forceinline__ void issue_rows(const DecodeParams& p, int b, int p0, const uint32_t* list, int e0,
                                           int rows, uint8_t* work, const Misc* misc) {
  constexpr int ROWB = D * (int)sizeof(T);
  constexpr int CPR = ROWB / 16;
  for (int i = threadIdx.x; i < rows * CPR; i += kThreads) {
    const int r = i / CPR, c = i % CPR;
    const uint32_t ent = list[e0 + r];
    const int vh = misc->gvh[ent >> 24];
    const uint8_t* src = reinterpret_cast<const uint8_t*>(reinterpret_cast<const T*>(p.v) + (int64_t)b * p.v_sb +
                                                          (int64_t)vh * p.v_sh +
                                                          (int64_t)(p0 + (int)(ent & 0xFFFFu)) * p.v_sl);
    cp_async16(work + (size_t)r * ROWB + c * 16, src + c * 16, true);
  }
  cp_async_commit();
}

template <typename T, int D, int MODE>
__device__ void gather_begin(const DecodeParams& p, int b, int h0, int p0, int n, const uint32_t* __restrict__ hmask,
                             uint32_t* __restrict__ list, int* __restrict__ tcnt, int* __restrict__ toff,
                             uint8_t* __restrict__ work, Misc* misc) {
  constexpr bool kDense = (MODE == MODE_DENSE);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, Gv = p.Gv, nw = (n + 31) / 32;
  const int vh_lo = h0 / Gv, vh_hi = (h0 + G - 1) / Gv;
  if (threadIdx.x == 0) {
    int ng = 0;
    for (int vh = vh_lo; vh <= vh_hi; ++vh) {
      const int a = max(h0, vh * Gv) - h0;
      const int bnd = min(h0 + G, (vh + 1) * Gv) - h0;
      for (int hb = a; hb < bnd && ng < kMaxGatherGroups; hb += 8) {
        misc->gvh[ng] = vh;
        misc->ghb[ng] = hb | (min(8, bnd - hb) << 16);
        ++ng;
      }
    }
    misc->ngroups = ng;
  }
  __syncthreads();
  const int ngroups = misc->ngroups;
  const int ntasks = ngroups * nw;
  // pass 1: entries per (group, 32-position word)
  for (int t = warp; t < ntasks; t += kWarps) {
    const int gi = t / nw, ww = t - gi * nw;
    const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
    const uint32_t gm = ((1u << nh) - 1u) << hb;
    const int pos = ww * 32 + lane;
    const bool has = pos < n && (kDense || (hmask[pos] & gm) != 0u);
    const uint32_t bal = __ballot_sync(0xffffffffu, has);
    if (lane == 0) tcnt[t] = __popc(bal);
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan in task order
    int run = 0;
    for (int b0 = 0; b0 < ntasks; b0 += 32) {
      const int t = b0 + lane;
      const int c = t < ntasks ? tcnt[t] : 0;
      const int incl = warp_incl_scan(c);
      if (t < ntasks) toff[t] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) misc->gstart[ngroups] = run;
  }
  __syncthreads();
  for (int gi = threadIdx.x; gi < ngroups; gi += kThreads) misc->gstart[gi] = toff[gi * nw];
  // pass 2: the entries
  for (int t = warp; t < ntasks; t += kWarps) {
    const int gi = t / nw, ww = t - gi * nw;
    const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
    const uint32_t gm = ((1u << nh) - 1u) << hb;
    const int pos = ww * 32 + lane;
    const uint32_t hm = pos < n ? (kDense ? gm : (hmask[pos] & gm)) : 0u;
    const uint32_t bal = __ballot_sync(0xffffffffu, hm != 0u);
    if (hm) list[toff[t] + __popc(bal & ((1u << lane) - 1u))] = (uint32_t)pos | ((hm >> hb) << 16) | ((uint32_t)gi << 24);
  }
  __syncthreads();
  if (p.trace && threadIdx.x == 0 && blockIdx.x < 1024) p.trace[blockIdx.x * 64 + 5] = clock64();
  const int total = misc->gstart[ngroups];
  if (total > 0 && total <= p.sm.br) issue_rows<T, D>(p, b, p0, list, 0, total, work, misc);
}

template <typename T, int D, int MODE>
__device__ void gather_end(const DecodeParams& p, int g, int j, int b, int h0, int p0, int n,
                           const T* __restrict__ sc, const uint32_t* __restrict__ hmask,
                           const uint32_t* __restrict__ list, uint8_t* __restrict__ work, float* __restrict__ wbuf,
                           Misc* misc) {
  constexpr int EPL = D / 32;
  constexpr int ROWB = D * (int)sizeof(T);
  constexpr bool kDense = (MODE == MODE_DENSE);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, SH = p.sh;
  const int BR = p.sm.br;
  const uint32_t tag = misc->tag;
  const int ngroups = misc->ngroups;
  const int total = misc->gstart[ngroups];
  const bool one_batch = total <= BR;

  auto weights = [&](int e0, int rows) {
    for (int i = threadIdx.x; i < rows * 8; i += kThreads) {
      const int r = i >> 3, hh = i & 7;
      const uint32_t ent = list[e0 + r];
      const int gi = ent >> 24;
      const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
      const int pos = ent & 0xFFFFu;
      float wv = 0.f;
      if (hh < nh && (kDense || ((hmask[pos] >> (hb + hh)) & 1u))) wv = weight_of<T, MODE>(sc, SH, misc, hb + hh, pos);
      wbuf[i] = wv;
    }
  };
  const bool tr = p.trace && threadIdx.x == 0 && blockIdx.x < 1024;
  if (tr) p.trace[blockIdx.x * 64 + 63] = total;
  if (one_batch && total > 0) {
    weights(0, total);
    cp_async_wait<0>();
    __syncthreads();
  }
  if (tr) p.trace[blockIdx.x * 64 + 12] = clock64();

  for (int gi = 0; gi < ngroups; ++gi) {
    const int g0 = misc->gstart[gi], g1 = misc->gstart[gi + 1];
    const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
    float acc[8][EPL];
    float accl[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      accl[i] = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[i][e] = 0.f;
    }
    for (int e0 = g0; e0 < g1; e0 += BR) {
      const int rows = min(BR, g1 - e0);
      int rbase = e0;  // SMEM row of entry e0
      if (!one_batch) {
        issue_rows<T, D>(p, b, p0, list, e0, rows, work, misc);
        weights(e0, rows);
        cp_async_wait<0>();
        __syncthreads();
        rbase = 0;
      }
      for (int r = warp; r < rows; r += kWarps) {
        const int rr = rbase + r;
        float vf[EPL];
        loadNf<T, EPL>(reinterpret_cast<const T*>(work + (size_t)rr * ROWB) + lane * EPL, vf);
        const float4 wa = *reinterpret_cast<const float4*>(wbuf + rr * 8);
        const float4 wb = *reinterpret_cast<const float4*>(wbuf + rr * 8 + 4);
        const float wr[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) {
          accl[hh] += wr[hh];
#pragma unroll
          for (int i = 0; i < EPL; ++i) acc[hh][i] = fmaf(wr[hh], vf[i], acc[hh][i]);
        }
      }
      if (!one_batch) __syncthreads();
    }
    if (tr && gi == 0) p.trace[blockIdx.x * 64 + 13] = clock64();
    // cross-warp reduction in a fixed order, one head at a time, in the SMEM
    // past the resident rows' weights
    float* red = wbuf + (size_t)BR * 8;  // [kWarps][D + 1]
    for (int hh = 0; hh < nh; ++hh) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k == hh) {
#pragma unroll
          for (int i = 0; i < EPL; ++i) red[warp * (D + 1) + lane * EPL + i] = acc[k][i];
          if (lane == 0) red[warp * (D + 1) + D] = accl[k];
        }
      }
      __syncthreads();
      for (int d = threadIdx.x; d <= D; d += kThreads) {
        float s = 0.f;
#pragma unroll
        for (int wp = 0; wp < kWarps; ++wp) s += red[wp * (D + 1) + d];
        slot_put(slot_at(p, g, j, hb + hh, d < D ? kSlotO + d : kSlotL), tag, __float_as_uint(s));
      }
      __syncthreads();
    }
  }
  for (int hl = threadIdx.x; hl < G; hl += kThreads)
    slot_put(slot_at(p, g, j, hl, kSlotM), tag, __float_as_uint(MODE == MODE_CALIBRATE ? 0.f : misc->aux[hl]));
  if (tr) p.trace[blockIdx.x * 64 + 14] = clock64();
}

// ---------------------------------------------------------------------------
// Merge of the group's partials: chunk j produces outputs [lo, hi) of the
// flattened (local head, d) space. All the partials it needs are fetched in
// one burst; sums run in chunk order.
// ---------------------------------------------------------------------------
template <typename T, int D, int MODE>
__device__ void merge_slice(const DecodeParams& p, int g, int j, int b, int h0, uint8_t* scratch, Misc* misc) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, C = p.C;
  const int tot = G * D;
  const int per = (tot + C - 1) / C;
  const int lo = j * per, hi = min(tot, lo + per);
  if (lo >= hi) return;
  const int hl0 = lo / D, hl1 = (hi - 1) / D;
  const int nhs = hl1 - hl0 + 1;
  const int nout = hi - lo;
  const uint32_t tag = misc->tag;
  uint32_t* ml = reinterpret_cast<uint32_t*>(scratch);  // [nhs][C][2]
  uint32_t* ov = ml + nhs * C * 2;                      // [nout][C]
  const int n_ml = nhs * C * 2;
  slots_gather(
      n_ml + nout * C,
      [&](int i) {
        if (i < n_ml) {
          const int hh = i / (2 * C), r = i % (2 * C);
          return slot_at(p, g, r >> 1, hl0 + hh, kSlotM + (r & 1));
        }
        const int k = i - n_ml;
        const int o = lo + k / C, c = k % C;
        return slot_at(p, g, c, o / D, kSlotO + o % D);
      },
      tag, ml, p.status);
  __syncthreads();
  if (p.trace && threadIdx.x == 0 && blockIdx.x < 1024) p.trace[blockIdx.x * 64 + 15] = clock64();
  float* scl = reinterpret_cast<float*>(ov + nout * C);  // [nhs][C]
  for (int hh = warp; hh < nhs; hh += kWarps) {
    float M = -INFINITY;
    for (int c = lane; c < C; c += 32) M = nanmax(M, __uint_as_float(ml[(hh * C + c) * 2]));
    M = warp_nanmax(M);
    float Ls = 0.f;
    for (int c = lane; c < C; c += 32) {
      const float mc = __uint_as_float(ml[(hh * C + c) * 2]);
      const float f = (MODE == MODE_CALIBRATE) ? 1.f : __expf(mc - M);
      scl[hh * C + c] = f;
      Ls += __uint_as_float(ml[(hh * C + c) * 2 + 1]) * f;
    }
    Ls = warp_sum(Ls);
    // calibration renormalises by max(sum p, 1e-12) (attention.py:161)
    if (lane == 0) misc->lsum[hh] = (MODE == MODE_CALIBRATE) ? fmaxf(Ls, 1e-12f) : Ls;
  }
  __syncthreads();
  for (int k = threadIdx.x; k < nout; k += kThreads) {
    const int o = lo + k;
    const int hh = o / D - hl0, d = o % D;
    float acc = 0.f;
    for (int c = 0; c < C; ++c) acc += __uint_as_float(ov[k * C + c]) * scl[hh * C + c];
    T* out = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)(h0 + o / D) * p.o_sh + d;
    *out = Num<T>::from_f(acc / misc->lsum[hh]);
  }
}

// Radix select: warp-parallel search of the bin holding the `want`-th largest
// key among 256 bins (bin 255 = largest). Returns the bin; *above = count in
// higher bins. Called by a full warp.
__device__ __forceinline__ int find_bin(const int* hist256, int want, int* above) {
  const int lane = threadIdx.x & 31;
  int c[8];
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = __ldcg(&hist256[255 - lane * 8 - i]);
    s += c[i];
  }
  const int incl = warp_incl_scan(s);
  const int before = incl - s;
  int bin = -1, ab = 0;
  if (before < want && want <= incl) {
    int cum = before;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (bin < 0) {
        if (cum + c[i] >= want) {
          bin = 255 - lane * 8 - i;
          ab = cum;
        }
        cum += c[i];
      }
    }
  }
  const unsigned bal = __ballot_sync(0xffffffffu, bin >= 0);
  if (bal == 0) {
    *above = 0;
    return 0;
  }
  const int src = __ffs(bal) - 1;
  bin = __shfl_sync(0xffffffffu, bin, src);
  *above = __shfl_sync(0xffffffffu, ab, src);
  return bin;
}

// ---------------------------------------------------------------------------
// The fused kernel.
// ---------------------------------------------------------------------------
template <typename T, int D, int MODE, bool TC, bool MASK>
__global__ void __launch_bounds__(kThreads, 1) saga_decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-aligned base (the 128-B swizzle pattern is taken from address bits)
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  Misc* misc = reinterpret_cast<Misc*>(smem + p.sm.misc);
  uint8_t* qop = smem + p.sm.qop;
  float* qf = reinterpret_cast<float*>(smem + p.sm.qop);
  T* sc = reinterpret_cast<T*>(smem + p.sm.scores);
  T* tsc = reinterpret_cast<T*>(smem + p.sm.tail);
  uint32_t* sel = reinterpret_cast<uint32_t*>(smem + p.sm.sel);
  uint32_t* eqb = reinterpret_cast<uint32_t*>(smem + p.sm.eq);
  uint32_t* list = reinterpret_cast<uint32_t*>(smem + p.sm.list);
  uint32_t* hmask = reinterpret_cast<uint32_t*>(smem + p.sm.hmask);
  int* tcnt = reinterpret_cast<int*>(smem + p.sm.sel);  // gather task counts (sel is free by then)
  int* toff = reinterpret_cast<int*>(smem + p.sm.eq);   // gather task offsets
  float* wbuf = reinterpret_cast<float*>(smem + p.sm.wbuf);
  uint8_t* work = smem + p.sm.work;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, C = p.C, CL = p.CL, SH = p.sh;
  Ring rg;
  uint32_t tmem_base = 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&misc->full[s], 1);
      mbar_init(&misc->empty[s], 1);
    }
    for (int bb = 0; bb < 2; ++bb) {
      mbar_init(&misc->tfull[bb], 1);
      mbar_init(&misc->tempty[bb], 4);
    }
    misc->abort = 0;
    mbar_fence_init();
  }
  if constexpr (TC) {
    if (warp == 1) tmem_alloc(&misc->tmem_slot, 32);
    tc_fence_before();
  }
  __syncthreads();
  if constexpr (TC) {
    tc_fence_after();
    tmem_base = misc->tmem_slot;
  }

  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int g = item / C, j = item % C;
    const int b = g / p.Hk, kh = g % p.Hk, h0 = kh * G;
    const int p0 = j * CL;
    const int n = min(p.L - p0, CL);
    const int nw = (n + 31) / 32;
    int* ctrl = p.ctrl + (size_t)g * kCtrlInts;
    ChunkStat* stg = p.stats + (size_t)g * C * G;  // [C][G] (calibration)
    ChunkStat* st = stg + (size_t)j * G;
    const int row0 = b * p.Hq + h0;
    const bool tracing = p.trace && threadIdx.x == 0 && item == (int)blockIdx.x && blockIdx.x < 1024;
#define SAGA_TRACE(k) \
  if (tracing) p.trace[blockIdx.x * 64 + (k)] = clock64();
    SAGA_TRACE(0)
    if constexpr (MODE != MODE_LOGITS) {  // the logits-only mode has no workspace
      if (threadIdx.x == 0) misc->tag = (uint32_t)ld_acquire_gpu(ctrl) + 1u;
    }

    // ---- fused append of the decode token (StaticLayer.update's index_copy_).
    // Every chunk of the group writes the new key row (the same values) before
    // it reads the cache, because every chunk scores the tail positions; the
    // chunk that owns the position also writes the value rows it gathers.
    if (p.k_new) {
      const int pos = p.append_pos;
      const T* src = reinterpret_cast<const T*>(p.k_new) + (int64_t)b * p.kn_sb + (int64_t)kh * p.kn_sh;
      T* dst = const_cast<T*>(reinterpret_cast<const T*>(p.k)) + (int64_t)b * p.k_sb + (int64_t)kh * p.k_sh +
               (int64_t)pos * p.k_sl;
      for (int d = threadIdx.x; d < D; d += kThreads) dst[d] = src[d];
      if (p.v_new && pos >= p0 && pos < p0 + n) {
        const int vh_lo = h0 / p.Gv, vh_hi = (h0 + G - 1) / p.Gv;
        for (int i = threadIdx.x; i < (vh_hi - vh_lo + 1) * D; i += kThreads) {
          const int vh = vh_lo + i / D, d = i % D;
          const T* vs = reinterpret_cast<const T*>(p.v_new) + (int64_t)b * p.vn_sb + (int64_t)vh * p.vn_sh;
          T* vd = const_cast<T*>(reinterpret_cast<const T*>(p.v)) + (int64_t)b * p.v_sb + (int64_t)vh * p.v_sh +
                  (int64_t)pos * p.v_sl;
          vd[d] = vs[d];
        }
      }
      __threadfence_block();
      fence_proxy_async_global();  // the appended rows are read back by TMA
    }

    // ---- logits of the chunk (and, for amortized, the tail max) ----
    const int tail_start = p.L - p.tail;
    if constexpr (TC) {
      int pre0 = 0, n_pre = 0;
      if (MODE == MODE_AMORTIZED) {
        pre0 = tail_start / kTile;
        n_pre = (p.L + kTile - 1) / kTile - pre0;
      }
      __syncthreads();
      score_chunk_tc<T, D, MODE, MASK>(p, b, kh, p0, n, pre0, n_pre, sc, tsc, qop, work, misc, rg, tmem_base);
      const int ej2 = (MODE == MODE_AMORTIZED) ? 2 * (((G + 1) / 2) / 2) : 0;
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        if (hl < ej2) {  // heads folded by the epilogue warps
          misc->s[hl] = ((misc->esum4[0][hl] + misc->esum4[1][hl]) + misc->esum4[2][hl]) + misc->esum4[3][hl];
          misc->aux[hl] = fmaxf(fmaxf(misc->emax4[0][hl], misc->emax4[1][hl]),
                                fmaxf(misc->emax4[2][hl], misc->emax4[3][hl]));
        } else {
          misc->s[hl] = misc->ered[0][hl] + misc->ered[1][hl];
          misc->aux[hl] = fmaxf(misc->emax[0][hl], misc->emax[1][hl]);  // chunk max
        }
      }
      __syncthreads();
    } else {
      for (int i = threadIdx.x; i < G * D; i += kThreads) {
        const int hl = i / D, d = i % D;
        qf[i] = Num<T>::to_f(reinterpret_cast<const T*>(p.q)[(int64_t)b * p.q_sb + (int64_t)(h0 + hl) * p.q_sh + d]);
      }
      for (int hl = threadIdx.x; hl < kMaxG; hl += kThreads) misc->tkey[hl] = 0u;
      __syncthreads();
      if (MODE == MODE_AMORTIZED)
        score_range_simt<T, D, MASK>(p, b, kh, tail_start, p.tail, p0, true, qf, sc, work, misc);
      score_range_simt<T, D, MASK>(p, b, kh, p0, n, p0, false, qf, sc, work, misc);
      for (int hl = warp; hl < G; hl += kWarps) {
        const float m = funkey(misc->tkey[hl]);
        float s = 0.f, mx = -INFINITY;
        for (int i = lane; i < n; i += 32) {
          const float l = Num<T>::to_f(sc[i * SH + hl]);
          if (MODE == MODE_AMORTIZED) s += exp_term<T>(l, m);
          mx = fmaxf(mx, l);
        }
        s = warp_sum(s);
        mx = warp_max(mx);
        if (lane == 0) {
          misc->m[hl] = m;
          misc->s[hl] = s;
          misc->aux[hl] = mx;
        }
      }
      __syncthreads();
    }
    SAGA_TRACE(1)

    if constexpr (MODE == MODE_LOGITS) {
      T* lo = reinterpret_cast<T*>(p.logits_out);
      for (int i = threadIdx.x; i < G * n; i += kThreads) {
        const int hl = i / n, pl = i % n;
        lo[(int64_t)(row0 + hl) * p.lo_ld + p0 + pl] = sc[pl * SH + hl];
      }
      __syncthreads();
      continue;
    }

    const uint32_t tag = misc->tag;
    uint32_t* xbuf = reinterpret_cast<uint32_t*>(smem + p.sm.xbuf);  // exchange staging [C][G]

    if constexpr (MODE == MODE_AMORTIZED) {
      // exchange the partial exp-sums (attention.py:145: sum over the row)
      for (int hl = threadIdx.x; hl < G; hl += kThreads)
        slot_put(slot_at(p, g, j, hl, kSlotS), tag, __float_as_uint(misc->s[hl]));
      slots_gather(C * G, [&](int i) { return slot_at(p, g, i / G, i % G, kSlotS); }, tag, xbuf, p.status);
      __syncthreads();
      SAGA_TRACE(2)
      // logit threshold t = m + log(max(thr, 1e-30) * s)  (attention.py:147)
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        float s = 0.f;
        for (int c = 0; c < C; ++c) s += __uint_as_float(xbuf[c * G + hl]);
        s = Num<T>::round(s);
        const float thr = clamp_min_keep_nan(p.thr_in[row0 + hl], 1e-30f);
        const float t = __fadd_rn(misc->m[hl], logf(__fmul_rn(thr, s)));
        misc->t[hl] = t;
        if (j == 0) {
          if (p.logit_thr_out) p.logit_thr_out[row0 + hl] = t;
          if (!isfinite(t)) set_status(p.status, SAGA_STATUS_NONFINITE_THR);
        }
      }
      __syncthreads();
      SAGA_TRACE(8)
      // strict selection x > t (triton_atopn.py:42): per position, the mask of
      // the heads it passes for, and per-thread per-head counts
      {
        float tl[kMaxG];
        int cnt[kMaxG];
#pragma unroll
        for (int hl = 0; hl < kMaxG; ++hl) {
          tl[hl] = (hl < G) ? misc->t[hl] : INFINITY;
          cnt[hl] = 0;
        }
        for (int i = threadIdx.x; i < n; i += kThreads) {
          uint32_t bits = 0;
#pragma unroll
          for (int hsb = 0; hsb < kMaxG / 16; ++hsb) {
            if (hsb * 16 < G) {
              float lv[16];
              const T* row = sc + (size_t)i * SH + hsb * 16;
              load8f<T>(row, lv);
              load8f<T>(row + 8, lv + 8);
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const bool pass = lv[k] > tl[hsb * 16 + k];  // false for padded slots (t = inf)
                bits |= (uint32_t)pass << (hsb * 16 + k);
                cnt[hsb * 16 + k] += pass;
              }
            }
          }
          hmask[i] = bits;
        }
#pragma unroll
        for (int hl = 0; hl < kMaxG; ++hl) {
          if (hl < G) {
            const int c = warp_sum_i(cnt[hl]);
            if (lane == 0) misc->cntw[warp][hl] = c;
          }
        }
      }
      __syncthreads();
      SAGA_TRACE(9)
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        int cnt = 0;
#pragma unroll
        for (int wp = 0; wp < kWarps; ++wp) cnt += misc->cntw[wp][hl];
        misc->i2[hl] = cnt;
        slot_put(slot_at(p, g, j, hl, kSlotCnt), tag, (uint32_t)cnt);
      }
      // lists and value-row copies go out while the counts are exchanged
      gather_begin<T, D, MODE>(p, b, h0, p0, n, hmask, list, tcnt, toff, work, misc);
      SAGA_TRACE(3)
      slots_gather(C * G, [&](int i) { return slot_at(p, g, i / G, i % G, kSlotCnt); }, tag, xbuf, p.status);
      __syncthreads();
      SAGA_TRACE(4)
      // exclusive prefix in chunk order: keep the K lowest passing positions
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        int pre = 0, tot = 0;
        for (int c = 0; c < C; ++c) {
          const int cc = (int)xbuf[c * G + hl];
          if (c < j) pre += cc;
          tot += cc;
        }
        const int mine = misc->i2[hl];
        pre = max(0, pre);  // bounds every offset below even if the slots were corrupt
        misc->i0[hl] = pre;
        misc->i1[hl] = max(0, min(mine, p.buf_k - pre));
        if (j == 0) {
          if (p.count_out) p.count_out[row0 + hl] = tot;
          if (tot > p.buf_k) set_status(p.status, SAGA_STATUS_OVERFLOW);
          if (tot == 0) set_status(p.status, SAGA_STATUS_EMPTY_ROW);
        }
      }
      __syncthreads();
      SAGA_TRACE(10)
      for (int hl = warp; hl < G; hl += kWarps) {
        if (misc->i1[hl] < misc->i2[hl]) {
          // capped chunk: clear this head's passing positions past K, and use
          // the max of the kept logits as the stabiliser
          const int keep = misc->i1[hl];
          int running = 0;
          float m = -INFINITY;
          for (int w = 0; w < nw; ++w) {
            const int i = w * 32 + lane;
            const bool on = i < n && ((hmask[i] >> hl) & 1u);
            const uint32_t bal = __ballot_sync(0xffffffffu, on);
            const int rank = running + __popc(bal & ((1u << lane) - 1u));
            if (on) {
              if (rank >= keep) atomicAnd(&hmask[i], ~(1u << hl));
              else m = fmaxf(m, Num<T>::to_f(sc[(size_t)i * SH + hl]));
            }
            running += __popc(bal);
          }
          m = warp_max(m);
          if (lane == 0) misc->aux[hl] = m;
        }
      }
      __syncthreads();
      if (p.sel_idx_out) {
        for (int hl = warp; hl < G; hl += kWarps) {
          int o = misc->i0[hl];
          const int lim = min(p.sel_ld, misc->i0[hl] + misc->i1[hl]);
          int* dst = p.sel_idx_out + (size_t)(row0 + hl) * p.sel_ld;
          for (int w = 0; w < nw && o < lim; ++w) {
            const int i = w * 32 + lane;
            const bool on = i < n && ((hmask[i] >> hl) & 1u);
            const uint32_t bal = __ballot_sync(0xffffffffu, on);
            const int k = o + __popc(bal & ((1u << lane) - 1u));
            if (on && k < lim) dst[k] = p0 + i;
            o += __popc(bal);
          }
        }
      }
      SAGA_TRACE(11)
      gather_end<T, D, MODE>(p, g, j, b, h0, p0, n, sc, hmask, list, work, wbuf, misc);
    } else if constexpr (MODE == MODE_CALIBRATE) {
      constexpr int KB = Num<T>::kKeyBits;
      constexpr int PASSES = KB / 8;
      const int nsel = p.buf_k;  // min(N, L)
      int* hsm = reinterpret_cast<int*>(work);     // [G][256]
      int* gh = p.hist + (size_t)g * 4 * G * 256;  // [pass][G][256]
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        st[hl].mx = misc->aux[hl];
        misc->i0[hl] = nsel;  // rank wanted within the current key prefix
        misc->i1[hl] = 0;     // key prefix so far
      }
      int sync_id = 2;
      for (int pass = 0; pass < PASSES; ++pass) {
        const int shift = KB - 8 * (pass + 1);
        for (int i = threadIdx.x; i < G * 256; i += kThreads) hsm[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < G * n; i += kThreads) {
          const int hl = i % G, pl = i / G;
          const uint32_t key = Num<T>::key(Num<T>::to_f(sc[pl * SH + hl]));
          const bool match = (pass == 0) || ((key >> (shift + 8)) == (uint32_t)misc->i1[hl]);
          if (match) atomicAdd(&hsm[hl * 256 + ((key >> shift) & 255u)], 1);
        }
        __syncthreads();
        for (int i = threadIdx.x; i < G * 256; i += kThreads)
          if (hsm[i]) atomicAdd(&gh[(size_t)pass * G * 256 + i], hsm[i]);
        if (pass == 1) {
          // exp-sum with the global max (attention.py:131-133 softmax)
          for (int hl = warp; hl < G; hl += kWarps) {
            const float M = misc->m[hl];
            float s = 0.f;
            for (int i = lane; i < n; i += 32) s += expf(__fsub_rn(Num<T>::to_f(sc[i * SH + hl]), M));
            s = warp_sum(s);
            if (lane == 0) st[hl].s = s;
          }
        }
        group_barrier(&ctrl[sync_id++], C, true, p.status, &misc->flag);
        if (pass == 0) {
          for (int hl = threadIdx.x; hl < G; hl += kThreads) {
            float M = -INFINITY;
            for (int c = 0; c < C; ++c) M = nanmax(M, __ldcg(&stg[(size_t)c * G + hl].mx));
            misc->m[hl] = M;
          }
        }
        if (pass == 1) {
          for (int hl = threadIdx.x; hl < G; hl += kThreads) {
            float s = 0.f;
            for (int c = 0; c < C; ++c) s += __ldcg(&stg[(size_t)c * G + hl].s);
            misc->s[hl] = s;
          }
        }
        for (int hl = warp; hl < G; hl += kWarps) {
          int above = 0;
          const int bin = find_bin(gh + (size_t)pass * G * 256 + hl * 256, misc->i0[hl], &above);
          if (lane == 0) {
            misc->i0[hl] -= above;
            misc->i1[hl] = (int)(((uint32_t)misc->i1[hl] << 8) | (uint32_t)bin);
          }
        }
        __syncthreads();
      }
      // the N-th largest logit; its probability is the threshold
      // (attention.py:181-187); softmax output exp(l - M) / S rounded.
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        const float lN = Num<T>::unkey((uint32_t)misc->i1[hl]);
        const float pN = Num<T>::round(__fdiv_rn(expf(__fsub_rn(lN, misc->m[hl])), misc->s[hl]));
        misc->t[hl] = lN;
        misc->aux[hl] = pN;
        if (j == 0 && p.thr_out) p.thr_out[row0 + hl] = pN;
      }
      __syncthreads();
      for (int hl = warp; hl < G; hl += kWarps) {
        const float M = misc->m[hl], S = misc->s[hl], pN = misc->aux[hl];
        int cg = 0, ce = 0;
        for (int w = 0; w < nw; ++w) {
          const int i = w * 32 + lane;
          float pr = 0.f;
          if (i < n) pr = Num<T>::round(__fdiv_rn(expf(__fsub_rn(Num<T>::to_f(sc[i * SH + hl]), M)), S));
          const uint32_t gb = __ballot_sync(0xffffffffu, (i < n) && pr > pN);
          const uint32_t eb = __ballot_sync(0xffffffffu, (i < n) && pr == pN);
          if (lane == 0) {
            sel[hl * (CL / 32) + w] = gb;
            eqb[hl * (CL / 32) + w] = eb;
          }
          cg += __popc(gb);
          ce += __popc(eb);
        }
        if (lane == 0) {
          st[hl].cnt = cg;
          st[hl].cnt_eq = ce;
          misc->i2[hl] = ce;
        }
      }
      group_barrier(&ctrl[sync_id++], C, true, p.status, &misc->flag);
      // ties at the N-th probability: the lowest positions fill the set
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        int tot_gt = 0;
        for (int c = 0; c < C; ++c) tot_gt += __ldcg(&stg[(size_t)c * G + hl].cnt);
        const int need = max(0, nsel - tot_gt);
        int eq_pre = 0, pos_pre = 0;
        for (int c = 0; c < j; ++c) {
          const int ce = __ldcg(&stg[(size_t)c * G + hl].cnt_eq);
          pos_pre += __ldcg(&stg[(size_t)c * G + hl].cnt) + max(0, min(ce, need - eq_pre));
          eq_pre += ce;
        }
        misc->i2[hl] = max(0, min(misc->i2[hl], need - eq_pre));  // kept ties here
        misc->i3[hl] = max(0, pos_pre);
        if (j == 0 && p.count_out) p.count_out[row0 + hl] = tot_gt;
      }
      __syncthreads();
      for (int hl = warp; hl < G; hl += kWarps) {
        warp_trim_bits(eqb + hl * (CL / 32), nw, misc->i2[hl]);
        for (int w = lane; w < nw; w += 32) sel[hl * (CL / 32) + w] |= eqb[hl * (CL / 32) + w];
        __syncwarp();
        if (p.sel_idx_out && misc->i3[hl] < p.sel_ld)
          warp_write_positions(sel + hl * (CL / 32), nw, p0,
                               p.sel_idx_out + (size_t)(row0 + hl) * p.sel_ld + misc->i3[hl],
                               max(0, p.sel_ld - misc->i3[hl]));
      }
      __syncthreads();
      for (int i = threadIdx.x; i < n; i += kThreads) {
        uint32_t bits = 0;
        for (int hl = 0; hl < G; ++hl) bits |= ((sel[hl * (CL / 32) + (i >> 5)] >> (i & 31)) & 1u) << hl;
        hmask[i] = bits;
      }
      __syncthreads();
      gather_begin<T, D, MODE>(p, b, h0, p0, n, hmask, list, tcnt, toff, work, misc);
      gather_end<T, D, MODE>(p, g, j, b, h0, p0, n, sc, hmask, list, work, wbuf, misc);
    } else {  // MODE_DENSE: misc->aux holds the chunk max from the scoring pass
      gather_begin<T, D, MODE>(p, b, h0, p0, n, hmask, list, tcnt, toff, work, misc);
      gather_end<T, D, MODE>(p, g, j, b, h0, p0, n, sc, hmask, list, work, wbuf, misc);
    }
    __syncthreads();

    // ---- merge of the group's partials, split across its chunks
    merge_slice<T, D, MODE>(p, g, j, b, h0, work, misc);
    SAGA_TRACE(6)

    // ---- the group's last chunk to finish advances the epoch and resets
    // the calibration counters and histograms
    __syncthreads();
    SAGA_TRACE(7)
#undef SAGA_TRACE
    if (threadIdx.x == 0) misc->last = (atomicAdd(&ctrl[kCtrlDone], 1) == C - 1);
    __syncthreads();
    if (misc->last) {
      if (threadIdx.x == 0) {
        ctrl[kCtrlDone] = 0;
        ctrl[0] = (int)tag;  // next launch's tag is tag + 1
      }
      for (int i = 1 + threadIdx.x; i < kCtrlDone; i += kThreads) ctrl[i] = 0;
      if (MODE == MODE_CALIBRATE) {
        int* gh = p.hist + (size_t)g * 4 * G * 256;
        for (int i = threadIdx.x; i < 4 * G * 256; i += kThreads) gh[i] = 0;
      }
    }
    __syncthreads();
  }

  if constexpr (TC) {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, 32);
    }
  }
}


// Kernel entry of one (dtype, head_dim, mode, scorer, mask) combination.
template <typename T, int D, int MODE, bool TC, bool MASK>
const void* decode_kernel_ptr() {
  return reinterpret_cast<const void*>(&saga_decode_kernel<T, D, MODE, TC, MASK>);
}

template <typename T, bool TC, bool MASK>
const void* pick_d_mode(int D, int mode) {
  if (D == 64) {
    switch (mode) {
      case MODE_AMORTIZED: return decode_kernel_ptr<T, 64, MODE_AMORTIZED, TC, MASK>();
      case MODE_CALIBRATE: return decode_kernel_ptr<T, 64, MODE_CALIBRATE, TC, MASK>();
      case MODE_DENSE: return decode_kernel_ptr<T, 64, MODE_DENSE, TC, MASK>();
      default: return decode_kernel_ptr<T, 64, MODE_LOGITS, TC, MASK>();
    }
  }
  switch (mode) {
    case MODE_AMORTIZED: return decode_kernel_ptr<T, 128, MODE_AMORTIZED, TC, MASK>();
    case MODE_CALIBRATE: return decode_kernel_ptr<T, 128, MODE_CALIBRATE, TC, MASK>();
    case MODE_DENSE: return decode_kernel_ptr<T, 128, MODE_DENSE, TC, MASK>();
    default: return decode_kernel_ptr<T, 128, MODE_LOGITS, TC, MASK>();
  }
}

}  // namespace saga
