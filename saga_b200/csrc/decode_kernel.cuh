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
  uint64_t tfull[kScoreBufs];  // TMEM accumulator ready (UMMA commit)
  uint64_t tempty[kScoreBufs]; // TMEM accumulator drained (4 epilogue warps)
  uint32_t tmem_slot;
  int abort;
  uint32_t tag;                // exchange tag of this launch for the current group
  int stored4[4];              // own tiles each epilogue warp stored to SMEM (this item)
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
  float aux2[kMaxG];   // merge: stabiliser of the combined partial per covered head
  float thr[kMaxG];     // softmax-space thresholds of the rows (amortized)
  int gstart[kMaxGatherGroups + 1];  // gather groups: list ranges
  int gvh[kMaxGatherGroups];         // gather group -> value head
  int ghb[kMaxGatherGroups];         // first local head | head count << 16
  uint32_t gmask[kMaxGatherGroups];  // local heads of the gather group as a bit mask
  int wsum[kWarps];                  // per-warp totals of a block scan
  int gpad[kMaxGatherGroups + 1];    // tensor-core P.V: first row slot of each gather group (16-aligned)
  float lacc[16 * 8];                // tensor-core P.V: weight sums per (gather group, head)
  uint64_t pvbar;                    // tensor-core P.V: a pass's MMAs completed
  uint64_t wfull[kMaxStages];        // dense P.V: a ring stage's weights written (4 epilogue warps)
  uint32_t vs0, vph0;                // dense P.V: ring stage and phase of its first value tile
  int ngroups;
  int flag;
  int last;
};
static_assert(sizeof(Misc) <= 6144, "Misc must fit its 6 KB slot");

// Paged caches: the page holding logical position pos of sequence b. A page
// number outside the pool sets SAGA_STATUS_PAGE_RANGE and page 0 is read.
__device__ __forceinline__ int page_of(const DecodeParams& p, int b, int pos) {
  int pg = __ldg(p.page_table + (int64_t)b * p.pt_sb + (pos >> p.page_shift));
  if ((unsigned)pg >= (unsigned)p.num_pages) {
    set_status(p.status, SAGA_STATUS_PAGE_RANGE);
    pg = 0;
  }
  return pg;
}
// Element offset of the row of (sequence b, head h, position pos) in a cache
// with strides (sb, sh, sl): contiguous, or inside page pg of a pool, sb then
// being the page stride.
template <bool PG>
__device__ __forceinline__ int64_t cache_row(const DecodeParams& p, int64_t sb, int64_t sh, int64_t sl, int b, int h,
                                             int pos, int pg) {
  if constexpr (PG) return (int64_t)pg * sb + (int64_t)h * sh + (int64_t)(pos & (p.page_len - 1)) * sl;
  else return (int64_t)b * sb + (int64_t)h * sh + (int64_t)pos * sl;
}
// Page of every 128-row tile of the item's chunk (paged caches), filled at
// item start; it sits in the same shared-memory carve as misc.
__device__ __forceinline__ int* tile_pages(const DecodeParams& p, const Misc* misc) {
  return reinterpret_cast<int*>(const_cast<uint8_t*>(reinterpret_cast<const uint8_t*>(misc)) - p.sm.misc + p.sm.tpg);
}
// TMA coordinates (row, outer) of the key tile at logical row y of sequence
// b: {y, b} for a contiguous cache; {row in page, page} for a paged one,
// own tile t >= 0 from the chunk's tile pages, a tail tile (t < 0) from the
// page table.
template <bool PG>
__device__ __forceinline__ void k_tile_coords(const DecodeParams& p, const Misc* misc, int b, int y, int t, int* ty,
                                              int* tw) {
  if constexpr (!PG) {
    *ty = y;
    *tw = b;
  } else {
    *tw = t >= 0 ? tile_pages(p, misc)[t] : page_of(p, b, y);
    *ty = y & (p.page_len - 1);
  }
}
// Element offset of the value row of head vh at chunk position r (chunks
// start on a tile boundary, so a tile lies in one page).
template <bool PG>
__device__ __forceinline__ int64_t value_row(const DecodeParams& p, const Misc* misc, int b, int vh, int p0, int r) {
  if constexpr (PG) return cache_row<true>(p, p.v_sb, p.v_sh, p.v_sl, b, vh, p0 + r, tile_pages(p, misc)[r >> 7]);
  else return cache_row<false>(p, p.v_sb, p.v_sh, p.v_sl, b, vh, p0 + r, 0);
}

template <int MODE>
__device__ __forceinline__ void item_prologue(const DecodeParams& p, int b, int kh, Misc* misc);

// Head pairs whose exp-sums the 4 epilogue warps fold while scoring (the 2
// helper warps take the rest): two thirds, which keeps both roles within one
// tile period (each helper warp covers twice the positions of an epilogue warp).
__device__ __forceinline__ int epilogue_exp_pairs(int G) { return (2 * ((G + 1) / 2) + 2) / 3; }

// Per-thread pipeline positions kept across items (only role threads use theirs).
struct Ring {
  uint32_t ps = 0, pph = 0;   // producer stage / phase
  uint32_t ms = 0, mph = 0;   // UMMA issuer stage / phase
  uint32_t mb = 0, mbph = 0;  // UMMA issuer TMEM buffer / phase
  uint32_t eb = 0, ebph = 0;  // epilogue TMEM buffer / phase
  uint32_t wpar = 0;          // UMMA issuer: next parity of each stage's wfull barrier (dense P.V)
};

// Optional phase trace (diagnostics), compiled in only when the library is
// built with SAGA_PHASE_TRACE=1: otherwise every stamp site compiles to
// nothing and SagaAttnArgs.trace is ignored (the stamp sites are many, and
// code size costs the latency-bound phases instruction fetches).
//  * trace_stamp(k), k < 16: SM clock at column k, global timer (ns,
//    comparable across SMs) at column 64 + k;
//  * trace_sub(k), k < 40: SM clock at column 80 + k, written by thread 0 of
//    CTA c < 1024 (its last item wins): where a phase spends its time;
//  * trace_col(col, v): raw value (columns 16-63 tile stamps, 120-122 global
//    timer at kernel entry, after set-up and at exit, 127 rows gathered).
#ifndef SAGA_PHASE_TRACE
#define SAGA_PHASE_TRACE 0
#endif
constexpr bool kTrace = SAGA_PHASE_TRACE != 0;
static __device__ __noinline__ void trace_write(long long* trace, int col, long long v) {
  trace[blockIdx.x * kTraceCols + col] = v;
}
static __device__ __noinline__ void trace_stamp_now(long long* trace, int k) {
  trace[blockIdx.x * kTraceCols + k] = clock64();
  trace[blockIdx.x * kTraceCols + 64 + k] = (long long)globaltimer_ns();
}
__device__ __forceinline__ void trace_stamp(const DecodeParams& p, int k) {
  if constexpr (kTrace)
    if (p.trace && blockIdx.x < 1024) trace_stamp_now(p.trace, k);
}
__device__ __forceinline__ void trace_sub(const DecodeParams& p, int k) {
  if constexpr (kTrace)
    if (p.trace && threadIdx.x == 0 && blockIdx.x < 1024) trace_write(p.trace, 80 + k, clock64());
}
__device__ __forceinline__ void trace_col(const DecodeParams& p, int col, long long v) {
  if constexpr (kTrace)
    if (p.trace && blockIdx.x < 1024) trace_write(p.trace, col, v);
}

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
// `pack_rd` rounds toward -inf: for any 16-bit value x and float t,
// x > t  <=>  x > round_down(t), so a threshold compare can run on pairs.
template <> struct Pair<__nv_bfloat16> {
  using P = __nv_bfloat162;
  __device__ __forceinline__ static P pack_rn(float a, float b) { return __floats2bfloat162_rn(a, b); }
  __device__ __forceinline__ static P pack_rd(float a, float b) {
    return __halves2bfloat162(__float2bfloat16_rd(a), __float2bfloat16_rd(b));
  }
  __device__ __forceinline__ static float2 unpack(P x) { return __bfloat1622float2(x); }
  __device__ __forceinline__ static P sub(P a, P b) { return __hsub2(a, b); }
  __device__ __forceinline__ static uint32_t gt_mask(P a, P b) { return __hgt2_mask(a, b); }
};
template <> struct Pair<__half> {
  using P = __half2;
  __device__ __forceinline__ static P pack_rn(float a, float b) { return __floats2half2_rn(a, b); }
  __device__ __forceinline__ static P pack_rd(float a, float b) {
    return __halves2half2(__float2half_rd(a), __float2half_rd(b));
  }
  __device__ __forceinline__ static float2 unpack(P x) { return __half22float2(x); }
  __device__ __forceinline__ static P sub(P a, P b) { return __hsub2(a, b); }
  __device__ __forceinline__ static uint32_t gt_mask(P a, P b) { return __hgt2_mask(a, b); }
};

// ---------------------------------------------------------------------------
// Epoch-tagged exchange slots
// ---------------------------------------------------------------------------
// Slots are read by the other CTAs of the group: GPU scope, or system scope
// when the sequence is sharded and the readers run on other devices (SHD).
template <bool SHD>
__device__ __forceinline__ void slot_put(unsigned long long* p, uint32_t tag, uint32_t bits) {
  const unsigned long long v = ((unsigned long long)tag << 32) | bits;
  if constexpr (SHD)
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
  else
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
template <bool SHD>
__device__ __forceinline__ unsigned long long slot_ld(const unsigned long long* p) {
  unsigned long long v;
  if constexpr (SHD)
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// All threads: fetch `count` slots (addresses from `addr(i)`) into dst[i].
// Each thread keeps up to 8 loads in flight (addresses computed once) and
// re-polls all of its pending slots together, so a late publisher costs one
// round trip, not one per slot. Bounded: after kWaitLimitNs the status word
// gets SAGA_STATUS_WAIT_TIMEOUT and the stale values are used.
template <bool SHD, int NT = kThreads, typename AddrFn>
__device__ __forceinline__ void slots_gather(int count, AddrFn addr, uint32_t tag, uint32_t* dst, int* status) {
  for (int base = threadIdx.x; base < count; base += NT * 8) {
    const unsigned long long* a[8];
    unsigned long long v[8];
    uint32_t pending = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + k * NT;
      a[k] = (i < count) ? addr(i) : nullptr;
      if (i < count) pending |= 1u << k;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = ((pending >> k) & 1u) ? slot_ld<SHD>(a[k]) : 0ull;
    unsigned long long t0 = 0;
#pragma unroll 1
    for (uint32_t it = 1;; ++it) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (((pending >> k) & 1u) && (uint32_t)(v[k] >> 32) == tag) {
          dst[base + k * NT] = (uint32_t)v[k];
          pending &= ~(1u << k);
        }
      }
      if (!pending) break;
      if ((it & 255u) == 0) {
        const unsigned long long now = globaltimer_ns();
        if (t0 == 0) {
          t0 = now;
        } else if (now - t0 > kWaitLimitNs) {
          if (status) atomicOr(status, SAGA_STATUS_WAIT_TIMEOUT);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            if ((pending >> k) & 1u) dst[base + k * NT] = (uint32_t)v[k];
          break;
        }
      }
      __nanosleep(32);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if ((pending >> k) & 1u) v[k] = slot_ld<SHD>(a[k]);
    }
  }
}

template <bool SHD>
__device__ __forceinline__ unsigned long long* slot_at(const DecodeParams& p, int g, int c, int hl, int k);
__device__ __forceinline__ unsigned long long* shard_slot(const DecodeParams& p, int g, int s, int hl, int k);

// Exchange of one per-(chunk, head) scalar field of group g over this
// device's chunks: dst[c * G + hl] for local chunk c (all of the group's
// chunks when the sequence is not sharded). One out-of-line copy serves
// every such exchange. NT threads take part.
template <bool SHD, int NT = kThreads>
static __device__ __noinline__ void slots_gather_field(const DecodeParams& p, int g, int field, uint32_t tag,
                                                       uint32_t* dst) {
  const FastDiv divg((uint32_t)p.G);
  const int c0 = SHD ? p.shard * p.c_local : 0;
  slots_gather<SHD, NT>(
      p.c_local * p.G,
      [&](int i) {
        const int c = (int)divg.div((uint32_t)i);
        return slot_at<SHD>(p, g, c0 + c, i - c * p.G, field);
      },
      tag, dst, p.status);
}
// The same field of every device's combined value: dst[s * G + hl].
static __device__ __noinline__ void slots_gather_shards(const DecodeParams& p, int g, int field, uint32_t tag,
                                                        uint32_t* dst) {
  const FastDiv divg((uint32_t)p.G);
  slots_gather<true>(
      p.shards * p.G,
      [&](int i) {
        const int sh = (int)divg.div((uint32_t)i);
        return shard_slot(p, g, sh, i - sh * p.G, field);
      },
      tag, dst, p.status);
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
template <typename T, int D, bool MASK, bool PG>
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
      const int pos = ok ? (a + s * SUB + r) : a;
      const T* src;
      if constexpr (PG)
        src = reinterpret_cast<const T*>(p.k) + cache_row<true>(p, p.k_sb, p.k_sh, p.k_sl, b, kh, pos, page_of(p, b, pos)) +
              cc * (16 / (int)sizeof(T));
      else
        src = kbase + (int64_t)pos * p.k_sl + cc * (16 / (int)sizeof(T));
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
template <typename T, int D, int MODE, bool MASK, bool PG>
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

  // The ring's stages are free at item start: the producer sends the first
  // tiles before the B operand is staged (the caller's barrier already made
  // the appended key row visible to TMA).
  int pre_issued = 0;
  if (warp == 0 && lane == 0) {
    for (int q = 0; q < min(NS, nseq); ++q) {
      if (!mbar_wait(&misc->empty[rg.ps], rg.pph ^ 1u, p.status)) {
        misc->abort = 1;
        break;
      }
      const int y = (q < n_pre) ? (pre0 + q) * 128 : p0 + (q - n_pre) * 128;
      int ty, tw;
      k_tile_coords<PG>(p, misc, b, y, q - n_pre, &ty, &tw);
      mbar_arrive_expect_tx(&misc->full[rg.ps], TILE_BYTES);
      uint8_t* dst = ring + rg.ps * TILE_BYTES;
#pragma unroll
      for (int kb = 0; kb < KB; ++kb)
        tma_load_4d(dst + kb * 16384, &p.tmap, kb * 64, ty, kh, tw, &misc->full[rg.ps]);
      if (q < 16) trace_col(p, 16 + q, clock64());
      ++pre_issued;
      if (++rg.ps == (uint32_t)NS) {
        rg.ps = 0;
        rg.pph ^= 1u;
      }
    }
  }
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
    for (int k = 0; k < 4; ++k) misc->stored4[k] = 0;
    misc->mready = 0;
    misc->tcount = 0;
  }
  fence_proxy_async_smem();
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      int issued = pre_issued;
      for (int q = pre_issued; q < nseq && !misc->abort; ++q) {
        if (!mbar_wait(&misc->empty[rg.ps], rg.pph ^ 1u, p.status)) {
          misc->abort = 1;
          break;
        }
        const int y = (q < n_pre) ? (pre0 + q) * 128 : p0 + (q - n_pre) * 128;
        int ty, tw;
        k_tile_coords<PG>(p, misc, b, y, q - n_pre, &ty, &tw);
        mbar_arrive_expect_tx(&misc->full[rg.ps], TILE_BYTES);
        uint8_t* dst = ring + rg.ps * TILE_BYTES;
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
          tma_load_4d(dst + kb * 16384, &p.tmap, kb * 64, ty, kh, tw, &misc->full[rg.ps]);
        ++issued;
        if (q < 16) trace_col(p, 16 + q, clock64());
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
        // descriptors of the tile's first K step, then constant offsets (the
        // start-address field counts 16-byte units): this warp shares its
        // scheduler with an epilogue warp, so few instructions per MMA
        const uint64_t ad0 = umma_desc_sw128(a0), bd0 = umma_desc_sw128(b0);
#pragma unroll
        for (int kb = 0; kb < KB; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16(dt, ad0 + (uint64_t)((kb * 16384 + kk * 32) >> 4), bd0 + (uint64_t)((kb * 2048 + kk * 32) >> 4),
                     IDESC, (kb | kk) != 0);
        umma_commit(&misc->empty[rg.ms]);
        umma_commit(&misc->tfull[rg.mb]);
        last_b = rg.mb;
        last_ph = rg.mbph;
        ++issued;
        if (q < 16) trace_col(p, 32 + q, clock64());
        if (++rg.ms == (uint32_t)NS) {
          rg.ms = 0;
          rg.mph ^= 1u;
        }
        if (++rg.mb == (uint32_t)kScoreBufs) {
          rg.mb = 0;
          rg.mbph ^= 1u;
        }
      }
      // all UMMAs of this item complete before their operands are reused
      if (issued) mbar_wait(&misc->tfull[last_b], last_ph, p.status);
      trace_col(p, 80 + 35, clock64());  // last tile's MMAs complete
    }
  } else if (warp >= 4) {
    // epilogue: TMEM -> logits (reference rounding chain) -> SMEM, 32 B per
    // position; for amortized it also folds the first EJ head pairs of its own
    // tiles into per-head exp-sums and maxima (the helpers take the rest)
    const int q4 = warp - 4;  // TMEM lane quarter of this warp
    const float scl = p.scaling;
    const int EJ = (MODE == MODE_AMORTIZED) ? epilogue_exp_pairs(G) : 0;
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
      if (++rg.eb == (uint32_t)kScoreBufs) {
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
      if (!pre && q - n_pre < 16 && q4 == 0 && lane == 0) trace_col(p, 48 + (q - n_pre), clock64());
      if (!pre && lane == 0) {
        __threadfence_block();
        atomicAdd(&misc->stored4[q4], 1);
      }
      if (pre && q == n_pre - 1) {
        // tail max of the group: warp max, then the last of the four epilogue
        // warps combines and publishes it (helpers and epilogue both wait)
        {
          const float v = warp_reduce16(tm, [](float x, float y) { return nanmax(x, y); });
          if ((lane & 1) == 0) misc->tmax4[q4][lane >> 1] = v;
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
    if (q4 == 0 && lane == 0) trace_col(p, 80 + 31, clock64());  // epilogue done with the tiles
    if (MODE == MODE_AMORTIZED) {
      const float sv = warp_reduce16(es, [](float x, float y) { return x + y; });
      const float mv = warp_reduce16(em, [](float x, float y) { return fmaxf(x, y); });
      const int k = lane >> 1;
      if ((lane & 1) == 0 && k < 2 * EJ) {
        misc->esum4[q4][k] = sv;
        misc->emax4[q4][k] = mv;
      }
    }
  } else if (warp == 2 || warp == 3) {
    // helpers: the item's exchange tag, gather groups and thresholds (their
    // global loads wait here, not in front of the scorer), then the per-head
    // exp-sum and maximum of every stored own tile
    const int hw = warp - 2;
    if constexpr (MODE != MODE_LOGITS) {
      if (warp == 3) item_prologue<MODE>(p, b, kh, misc);
    }
    float m[16], s[16], mx[16];
#pragma unroll
    for (int hl = 0; hl < 16; ++hl) {
      m[hl] = -INFINITY;
      s[hl] = 0.f;
      mx[hl] = -INFINITY;
    }
    // Tile q is complete once each of the four epilogue warps stored its
    // quarter: the warps may be a tile apart (two TMEM score buffers), so a
    // total over the warps could count a later tile of one warp instead.
    auto stored_min = [&]() {
      const volatile int* s4 = misc->stored4;
      return min(min(s4[0], s4[1]), min(s4[2], s4[3]));
    };
    auto wait_stored = [&](int target) {
      if (stored_min() >= target) return true;
      unsigned long long t0 = 0;
      for (uint32_t it = 1; stored_min() < target; ++it) {
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
    const int EJ = (MODE == MODE_AMORTIZED) ? epilogue_exp_pairs(G) : 0;
    P2 m2[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) m2[jj] = PT::pack_rn(m[2 * jj], m[2 * jj + 1]);
    for (int q = 0; q < ntl && live; ++q) {
      live = wait_stored(q + 1);
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
    if (lane == 0) trace_col(p, 80 + 32 + hw, clock64());  // helper warp done with the tiles
    {
      const float sv = warp_reduce16(s, [](float x, float y) { return x + y; });
      const float mv = warp_reduce16(mx, [](float x, float y) { return fmaxf(x, y); });
      const int hl = lane >> 1;
      if ((lane & 1) == 0 && hl < G) {
        misc->ered[hw][hl] = sv;
        misc->emax[hw][hl] = mv;
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
__device__ __forceinline__ float weight_from_logit(float l, const Misc* misc, int hl) {
  if constexpr (MODE == MODE_CALIBRATE) {
    return Num<T>::round(__fdiv_rn(expf(__fsub_rn(l, misc->m[hl])), misc->s[hl]));
  } else if constexpr (MODE == MODE_DENSE) {
    // A chunk the mask covers whole has max -inf; its weights are 0, not
    // exp(-inf - -inf). (Selected positions of the other modes are finite.)
    const float a = misc->aux[hl];
    return __expf(l - (a == -INFINITY ? 0.f : a));
  } else {
    return __expf(l - misc->aux[hl]);
  }
}
template <typename T, int MODE>
__device__ __forceinline__ float weight_of(const T* sc, int SH, const Misc* misc, int hl, int i) {
  return weight_from_logit<T, MODE>(Num<T>::to_f(sc[i * SH + hl]), misc, hl);
}

constexpr int kSlotS = 0, kSlotCnt = 1, kSlotM = 2, kSlotL = 3, kSlotO = 4;
// Slot k of head hl inside one record of G * (D + 4) slots: the scalar fields
// of every head first ([field][head]), then the partial outputs ([head][d]).
// An exchange of one field over the heads, and a merge slice of consecutive
// outputs of one chunk, then read consecutive slots (a few cache lines per
// warp instead of one per lane).
__device__ __forceinline__ size_t slot_in_record(int G, int D, int hl, int k) {
  return k < kSlotO ? (size_t)k * G + hl : (size_t)kSlotO * G + (size_t)hl * D + (k - kSlotO);
}
// Slot address: group g, chunk c, local head hl, field k.
template <bool SHD>
__device__ __forceinline__ unsigned long long* slot_at(const DecodeParams& p, int g, int c, int hl, int k) {
  int owner = 0;
  if constexpr (SHD) {  // chunk c of the group lives on shard c / c_local
    owner = c / p.c_local;
    c -= owner * p.c_local;
  }
  return p.slot_base[owner] + ((size_t)g * p.c_local + c) * p.G * (size_t)(p.D + 4) + slot_in_record(p.G, p.D, hl, k);
}

// Sequence sharding: the combined value of device s's chunks, in device s's
// workspace past the chunk slots: one record of G * (D + 4) per group.
__device__ __forceinline__ unsigned long long* shard_slot(const DecodeParams& p, int g, int s, int hl, int k) {
  const size_t chunk_slots = (size_t)p.B * p.Hk * p.c_local * p.G * (p.D + 4);
  return p.slot_base[s] + chunk_slots + (size_t)g * p.G * (p.D + 4) + slot_in_record(p.G, p.D, hl, k);
}

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
template <typename T, int D, bool PG>
__device__ __forceinline__ void issue_rows(const DecodeParams& p, int b, int p0, const uint32_t* list, int e0,
                                           int rows, uint8_t* work, const Misc* misc) {
  constexpr int ROWB = D * (int)sizeof(T);
  constexpr int CPR = ROWB / 16;
  for (int i = threadIdx.x; i < rows * CPR; i += kThreads) {
    const int r = i / CPR, c = i % CPR;
    const uint32_t ent = list[e0 + r];
    const int vh = misc->gvh[ent >> 24];
    const uint8_t* src = reinterpret_cast<const uint8_t*>(reinterpret_cast<const T*>(p.v) +
                                                          value_row<PG>(p, misc, b, vh, p0, (int)(ent & 0xFFFFu)));
    cp_async16(work + (size_t)r * ROWB + c * 16, src + c * 16, true);
  }
  cp_async_commit();
}

// Tensor-core P.V operand layouts (head_dim 128, 16-bit values):
//  * value rows: row slot s, 16-byte segment sg (8 elements) -> byte offset
//    in the MN-major 128-B swizzle layout: 8-slot groups of two 1024-B atoms
//    (elements 0-63 and 64-127 of the row), the segment index XOR-ed with s % 8;
//  * weights: slot s, head slot n < 16 -> byte offset in the K-major 128-B
//    swizzle layout: blocks of 64 slots x 16 head slots, one 128-B row per
//    head slot (only the group's heads are read back; see pv_weights).
__device__ __forceinline__ int pv_row_off(int s, int sg) {
  return (s >> 3) * 2048 + (sg >> 3) * 1024 + (s & 7) * 128 + (((sg & 7) ^ (s & 7)) << 4);
}
__device__ __forceinline__ int pv_w_off(int s, int n) {
  return (s >> 6) * 2048 + (n >> 3) * 1024 + (n & 7) * 128 + ((((s & 63) >> 3) ^ (n & 7)) << 4) + (s & 7) * 2;
}
// Gather group holding row slot s (groups are contiguous, ascending).
__device__ __forceinline__ int pv_group_of(const Misc* misc, int ngroups, int s) {
  int gi = 0;
  while (gi + 1 < ngroups && misc->gpad[gi + 1] <= s) ++gi;
  return gi;
}

// Copies of the value rows of global row slots [s0, s1) into pass slots
// s - pbase: rows of real entries from the cache, padding slots zero-filled.
// RPI = 2 rows per warp instruction, 16 segments each.
template <typename T, bool PG>
__device__ __noinline__ void pv_issue_rows(const DecodeParams& p, int b, int p0, const uint32_t* __restrict__ list,
                                              uint8_t* __restrict__ work, const Misc* misc, int ngroups, int s0,
                                              int s1, int pbase) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane >> 4, sg = lane & 15;
  const T* vb = reinterpret_cast<const T*>(p.v) + (int64_t)b * p.v_sb + (int64_t)p0 * p.v_sl;
  for (int gi = 0; gi < ngroups; ++gi) {
    const int a = max(misc->gpad[gi], s0), z = min(misc->gpad[gi + 1], s1);
    if (a >= z) continue;
    const int e0 = misc->gstart[gi], rows = misc->gstart[gi + 1] - e0, gbase = misc->gpad[gi];
    const T* vg = vb + (int64_t)misc->gvh[gi] * p.v_sh;
    if constexpr (PG) {  // paged: each row's page from the chunk's tile pages
      const T* v0 = reinterpret_cast<const T*>(p.v);
      for (int s = a + warp * 2 + sub; s < z; s += kWarps * 2) {
        const int r = s - gbase;
        uint8_t* dst = work + pv_row_off(s - pbase, sg);
        if (r < rows) {
          const int pos = (int)(list[e0 + r] & 0xFFFFu);
          cp_async16(dst, v0 + value_row<true>(p, misc, b, misc->gvh[gi], p0, pos) + sg * 8, true);
        } else {
          cp_async16(dst, v0, false);
        }
      }
      continue;
    }
#pragma unroll 2
    for (int s = a + warp * 2 + sub; s < z; s += kWarps * 2) {
      const int r = s - gbase;
      uint8_t* dst = work + pv_row_off(s - pbase, sg);
      if (r < rows) {
        const int pos = (int)(list[e0 + r] & 0xFFFFu);
        cp_async16(dst, vg + (int64_t)pos * p.v_sl + sg * 8, true);
      } else {
        cp_async16(dst, vg, false);  // zero row: padding of the 16-row MMA step
      }
    }
  }
}

// Weights of the P.V operand for pass slots [0, pn) (global slots ps0 + ...):
// one task per (8-slot chunk, head slot < 8) computes 8 weights and stores
// them as one 16-byte K-major segment; padding slots and unselected (row,
// head) pairs get 0. Only the MMA output columns of real heads are read, so
// head slots past the group's heads are left as they are, and the second half
// of each 64-slot block (head slots 8-15) holds the 8-weight partial sums:
// float at block + 1024 + chunk * 32 + head * 4. With `capped_only`, only the
// heads whose chunk was capped at K (keep < passing) are recomputed.
template <typename T, int MODE>
__device__ __noinline__ void pv_weights(const DecodeParams& p, const T* __restrict__ sc, const uint32_t* __restrict__ hmask,
                           const uint32_t* __restrict__ list, uint8_t* __restrict__ wpv, const Misc* misc,
                           int ngroups, int ps0, int pn, bool capped_only) {
  constexpr bool kDense = (MODE == MODE_DENSE);
  const int SH = p.sh;
  for (int i = threadIdx.x; i < (pn >> 3) * 8; i += kThreads) {
    const int c8 = i >> 3, nn = i & 7;
    const int ps = c8 * 8, gs = ps0 + ps;
    const int gi = pv_group_of(misc, ngroups, gs);
    const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
    const int hl = hb + nn;
    if (nn >= nh) continue;
    if (capped_only && misc->i1[hl] >= misc->i2[hl]) continue;
    const int e0 = misc->gstart[gi], rows = misc->gstart[gi + 1] - e0;
    const int r0 = gs - misc->gpad[gi];
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    float psum = 0.f;
    if (r0 < rows) {
      // all loads first (indices clamped to a real row), so the 8 chains overlap
      int pos[8];
      uint32_t hm[8];
      float l[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) pos[k] = (int)(list[e0 + min(r0 + k, rows - 1)] & 0xFFFFu);
      if constexpr (!kDense) {
#pragma unroll
        for (int k = 0; k < 8; ++k) hm[k] = hmask[pos[k]];
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) l[k] = Num<T>::to_f(sc[pos[k] * SH + hl]);
      T* e = reinterpret_cast<T*>(&u);
      float wr[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const bool on = (r0 + k < rows) && (kDense || ((hm[k] >> hl) & 1u));
        e[k] = Num<T>::from_f(on ? weight_from_logit<T, MODE>(l[k], misc, hl) : 0.f);
        wr[k] = Num<T>::to_f(e[k]);  // the rounded weight the MMA multiplies
      }
      psum = ((wr[0] + wr[1]) + (wr[2] + wr[3])) + ((wr[4] + wr[5]) + (wr[6] + wr[7]));
    }
    *reinterpret_cast<uint4*>(wpv + pv_w_off(ps, nn)) = u;
    *reinterpret_cast<float*>(wpv + (ps >> 6) * 2048 + 1024 + ((ps & 63) >> 3) * 32 + nn * 4) = psum;
  }
}

__device__ __forceinline__ void plan_gather_groups(const DecodeParams& p, int h0, Misc* misc);

// Per-item set-up done by one warp (the logits-only mode has no workspace):
// the exchange tag of this launch, the gather groups, and for amortized the
// rows' softmax-space thresholds.
template <int MODE>
__device__ __forceinline__ void item_prologue(const DecodeParams& p, int b, int kh, Misc* misc) {
  const int lane = threadIdx.x & 31;
  const int G = p.G, h0 = kh * G;
  if (lane == 0) {
    misc->tag = (uint32_t)ld_acquire_gpu(p.ctrl + (size_t)(b * p.Hk + kh) * kCtrlInts) + 1u;
    plan_gather_groups(p, h0, misc);
  }
  if (MODE == MODE_AMORTIZED && lane < G) misc->thr[lane] = p.thr_in[b * p.Hq + h0 + lane];
}

// Gather groups of an item: (value head, <= 8 of its query heads in this key
// group). One thread.
__device__ __forceinline__ void plan_gather_groups(const DecodeParams& p, int h0, Misc* misc) {
  const int G = p.G, Gv = p.Gv;
  const int vh_lo = h0 / Gv, vh_hi = (h0 + G - 1) / Gv;
  int ng = 0;
  for (int vh = vh_lo; vh <= vh_hi; ++vh) {
    const int a = max(h0, vh * Gv) - h0;
    const int bnd = min(h0 + G, (vh + 1) * Gv) - h0;
    for (int hb = a; hb < bnd && ng < kMaxGatherGroups; hb += 8) {
      const int nh = min(8, bnd - hb);
      misc->gvh[ng] = vh;
      misc->ghb[ng] = hb | (nh << 16);
      misc->gmask[ng] = ((1u << nh) - 1u) << hb;
      ++ng;
    }
  }
  misc->ngroups = ng;
}

// Strict selection of one chunk: hmask[i] = heads whose logit at position i
// exceeds misc->t (bit hl = local head hl), for i < nw * 32 (zero past n), and
// misc->cntw[warp][hl] = the warp's count of passing positions of head hl.
template <typename T>
__device__ __forceinline__ void select_heads(const T* __restrict__ sc, int SH, int G, int n, int nw, Misc* misc,
                                             uint32_t* __restrict__ hmask) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if constexpr (sizeof(T) == 2) {
    // pairs of heads per compare; counts packed two per word (16-bit halves)
    using PT = Pair<T>;
    using P = typename PT::P;
    P t2[16];
    uint32_t c2[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const float ta = (2 * k < G) ? misc->t[2 * k] : INFINITY;  // padded slots never pass
      const float tb = (2 * k + 1 < G) ? misc->t[2 * k + 1] : INFINITY;
      t2[k] = PT::pack_rd(ta, tb);
      c2[k] = 0u;
    }
    const int npairs = SH / 2;
    for (int i = threadIdx.x; i < nw * 32; i += kThreads) {
      uint32_t bits = 0;
      if (i < n) {
#pragma unroll
        for (int hsb = 0; hsb < 2; ++hsb) {
          if (hsb * 8 < npairs) {
            const uint4* row = reinterpret_cast<const uint4*>(sc + (size_t)i * SH + hsb * 16);
            const uint4 u0 = row[0], u1 = row[1];
            const P* pa = reinterpret_cast<const P*>(&u0);
            const P* pb = reinterpret_cast<const P*>(&u1);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t m = PT::gt_mask(k < 4 ? pa[k] : pb[k - 4], t2[hsb * 8 + k]) & 0x00010001u;
              c2[hsb * 8 + k] += m;
              bits |= ((m | (m >> 15)) & 3u) << (hsb * 16 + 2 * k);
            }
          }
        }
      }
      hmask[i] = bits;
    }
    {
      const uint32_t c = warp_reduce16(c2, [](uint32_t x, uint32_t y) { return x + y; });
      const int k = lane >> 1;  // head pair of this lane
      if ((lane & 1) == 0) {
        if (2 * k < G) misc->cntw[warp][2 * k] = (int)(c & 0xFFFFu);
        if (2 * k + 1 < G) misc->cntw[warp][2 * k + 1] = (int)(c >> 16);
      }
    }
  } else {
    float tl[kMaxG];
    int cnt[kMaxG];
#pragma unroll
    for (int hl = 0; hl < kMaxG; ++hl) {
      tl[hl] = (hl < G) ? misc->t[hl] : INFINITY;
      cnt[hl] = 0;
    }
    for (int i = threadIdx.x; i < nw * 32; i += kThreads) {
      uint32_t bits = 0;
      if (i < n) {
#pragma unroll
        for (int hsb = 0; hsb < kMaxG / 16; ++hsb) {
          if (hsb * 16 < SH) {
            float lv[16];
            const T* row = sc + (size_t)i * SH + hsb * 16;
            load8f<T>(row, lv);
            load8f<T>(row + 8, lv + 8);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const bool pass = lv[k] > tl[hsb * 16 + k];
              bits |= (uint32_t)pass << (hsb * 16 + k);
              cnt[hsb * 16 + k] += pass;
            }
          }
        }
      }
      hmask[i] = bits;
    }
    {
      int lo[16], hi[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        lo[k] = cnt[k];
        hi[k] = cnt[16 + k];
      }
      const auto add = [](int x, int y) { return x + y; };
      const int cl = warp_reduce16(lo, add);
      const int ch = (SH > 16) ? warp_reduce16(hi, add) : 0;
      const int k = lane >> 1;
      if ((lane & 1) == 0) {
        if (k < G) misc->cntw[warp][k] = cl;
        if (16 + k < G) misc->cntw[warp][16 + k] = ch;
      }
    }
  }
}

// Occupancy of one (gather group, 32-position word) task: bit k set if
// position w*32+k belongs to the group's list. hmask is zero past n.
template <bool kDense>
__device__ __forceinline__ uint32_t task_occupancy(const uint32_t* __restrict__ hmask, uint32_t gm, int w, int n) {
  if constexpr (kDense) {
    const int rem = n - w * 32;
    return rem >= 32 ? 0xffffffffu : ((1u << rem) - 1u);
  } else {
    const uint4* h4 = reinterpret_cast<const uint4*>(hmask + w * 32);
    uint32_t occ = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int c = (k + threadIdx.x) & 7;  // rotated so that neighbouring threads hit distinct banks
      const uint4 v = h4[c];
      occ |= ((uint32_t)((v.x & gm) != 0u) | ((uint32_t)((v.y & gm) != 0u) << 1) |
              ((uint32_t)((v.z & gm) != 0u) << 2) | ((uint32_t)((v.w & gm) != 0u) << 3))
             << (4 * c);
    }
    return occ;
  }
}

// TCPV: the kernel runs the tensor-core P.V (16-bit types at head_dim 128 on
// the tensor-core scorer); otherwise the CUDA-core P.V's rows are issued here
// when they fit one batch.
template <typename T, int D, int MODE, bool TCPV, bool PG>
__device__ void gather_begin(const DecodeParams& p, int b, int p0, int n, const T* __restrict__ sc,
                             const uint32_t* __restrict__ hmask, uint32_t* __restrict__ list, int* __restrict__ toff,
                             uint32_t* __restrict__ occ, uint8_t* __restrict__ work, uint8_t* __restrict__ wpv,
                             Misc* misc) {
  constexpr bool kDense = (MODE == MODE_DENSE);
  constexpr int ROWB = D * (int)sizeof(T);
  constexpr int CPR = ROWB / 16;      // 16-byte copies per value row (8, 16 or 32)
  constexpr int RPI = 32 / CPR;       // rows one warp copies per instruction
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (n + 31) / 32;
  const int ngroups = misc->ngroups;
  const int ntasks = ngroups * nw;
  // one (gather group, word) task per thread: occupancy, then an exclusive
  // scan of the counts in task order
  int carry = 0;
  trace_sub(p, 0);
  for (int t0 = 0; t0 < ntasks; t0 += kThreads) {
    const int t = t0 + threadIdx.x;
    int c = 0;
    if (t < ntasks) {
      const int gi = t / nw, w = t - gi * nw;
      const uint32_t o = task_occupancy<kDense>(hmask, misc->gmask[gi], w, n);
      occ[t] = o;
      c = __popc(o);
    }
    trace_sub(p, 1);
    const int incl = warp_incl_scan(c);
    if (lane == 31) misc->wsum[warp] = incl;
    __syncthreads();
    trace_sub(p, 2);
    int wpre = 0, tot = 0;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) {
      const int ws = misc->wsum[k];
      wpre += (k < warp) ? ws : 0;
      tot += ws;
    }
    if (t < ntasks) toff[t] = carry + wpre + incl - c;
    carry += tot;
    __syncthreads();
  }
  trace_sub(p, 3);
  // entries in ascending position order within each task
  for (int t = threadIdx.x; t < ntasks; t += kThreads) {
    uint32_t o = occ[t];
    if (!o) continue;
    const int gi = t / nw, w = t - gi * nw;
    const uint32_t gm = misc->gmask[gi];
    const int hb = misc->ghb[gi] & 0xFFFF;
    int e = toff[t];
    while (o) {
      const int bit = __ffs(o) - 1;
      o &= o - 1u;
      const int pos = w * 32 + bit;
      const uint32_t hm = kDense ? gm : (hmask[pos] & gm);
      list[e++] = (uint32_t)pos | ((hm >> hb) << 16) | ((uint32_t)gi << 24);
    }
  }
  trace_sub(p, 4);
  for (int gi = threadIdx.x; gi <= ngroups; gi += kThreads) {
    misc->gstart[gi] = gi < ngroups ? toff[gi * nw] : carry;
    if constexpr (TCPV) {
      int s = 0;  // row slots of the groups before gi, each group padded to 16
      for (int k = 0; k < gi; ++k) {
        const int e1 = (k + 1 < ngroups) ? toff[(k + 1) * nw] : carry;
        s += (e1 - toff[k * nw] + 15) & ~15;
      }
      misc->gpad[gi] = s;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(p, 5);
  if constexpr (TCPV && MODE == MODE_AMORTIZED) {
    // the first pass's weights before its row copies: the copies then do not
    // hold up these shared-memory reads
    pv_weights<T, MODE>(p, sc, hmask, list, wpv, misc, ngroups, 0, min(misc->gpad[ngroups], p.sm.brw), false);
    trace_sub(p, 5);
  }
  if constexpr (TCPV) {
    if (p.sm.brw > 0) {  // tensor-core P.V: the first pass's rows
      pv_issue_rows<T, PG>(p, b, p0, list, work, misc, ngroups, 0, min(misc->gpad[ngroups], p.sm.brw), 0);
      cp_async_commit();
      trace_sub(p, 6);
    }
    return;
  }
  // value rows, when they all fit one batch: RPI rows per warp instruction,
  // each row read as CPR consecutive 16-byte segments
  if (carry > 0 && carry <= p.sm.br) {
    const int sub = lane / CPR, seg = lane % CPR;
    const T* vb = reinterpret_cast<const T*>(p.v) + (int64_t)b * p.v_sb + (int64_t)p0 * p.v_sl;
#pragma unroll 2
    for (int e = warp * RPI + sub; e < carry; e += kWarps * RPI) {
      const uint32_t ent = list[e];
      const T* src;
      if constexpr (PG)
        src = reinterpret_cast<const T*>(p.v) + value_row<true>(p, misc, b, misc->gvh[ent >> 24], p0, (int)(ent & 0xFFFFu));
      else
        src = vb + (int64_t)misc->gvh[ent >> 24] * p.v_sh + (int64_t)(ent & 0xFFFFu) * p.v_sl;
      cp_async16(work + (size_t)e * ROWB + seg * 16, reinterpret_cast<const uint8_t*>(src) + seg * 16, true);
    }
  }
  cp_async_commit();
}

// Tensor-core P.V of one item (16-bit values, head_dim 128). Per pass of at
// most brw row slots: rows beyond the first pass are fetched now; the weights
// (rounded to the value type) go to the K-major operand; the MMA issuer
// accumulates out^T[d][head slot] += V^T[d][slot] * W[slot][head slot] into 16
// TMEM columns per gather group. The partial (m, l, o[D]) of every head is
// then published through the group's tagged slots.
template <typename T, int D, int MODE, bool SHD, bool PG>
__device__ void gather_end_tc(const DecodeParams& p, int g, int j, int b, int p0, const T* __restrict__ sc,
                              const uint32_t* __restrict__ hmask, const uint32_t* __restrict__ list,
                              uint8_t* __restrict__ work, uint8_t* __restrict__ wpv, Misc* misc, uint32_t tmem_base,
                              uint32_t& pvph, bool w0_ready) {
  constexpr bool kDense = (MODE == MODE_DENSE);
  constexpr uint32_t kIdesc = umma_idesc_f16(Num<T>::kDType == SAGA_BF16 ? 1u : 0u, 128, 16) | kUmmaAMajorMN;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, SH = p.sh, brw = p.sm.brw;
  const uint32_t tag = misc->tag;
  const int ngroups = misc->ngroups;
  const int TS = misc->gpad[ngroups];
  // accumulators per gather group: as many as the TMEM columns allow, at most 4
  const int nch = min(4, p.tmem_cols / (16 * max(ngroups, 1)));
  const bool tr = kTrace && p.trace && threadIdx.x == 0 && blockIdx.x < 1024;
  if (tr) trace_col(p, 127, misc->gstart[ngroups]);
  for (int t = threadIdx.x; t < ngroups * 8; t += kThreads) misc->lacc[t] = 0.f;
  if (brw < 16) {  // unreachable by construction of the layout; no pass could run
    if (threadIdx.x == 0) set_status(p.status, SAGA_STATUS_WAIT_TIMEOUT);
    return;
  }
  for (int ps0 = 0; ps0 < TS; ps0 += brw) {
    const int pn = min(brw, TS - ps0);
    if (ps0 > 0) {
      pv_issue_rows<T, PG>(p, b, p0, list, work, misc, ngroups, ps0, ps0 + pn, ps0);
      cp_async_commit();
    }
    if (!(ps0 == 0 && w0_ready)) pv_weights<T, MODE>(p, sc, hmask, list, wpv, misc, ngroups, ps0, pn, false);
    if (ps0 == 0) trace_sub(p, 10);
    cp_async_wait<0>();
    if (ps0 == 0) trace_sub(p, 11);
    fence_proxy_async_smem();  // weights and rows -> visible to the tensor cores
    tc_fence_before();
    __syncthreads();
    if (tr && ps0 == 0) trace_stamp(p, 12);
    if (warp == 1 && lane == 0) {
      tc_fence_after();
      const uint64_t ad0 = umma_desc_mn_sw128(smem_addr(work), 1024, 2048);
      const uint64_t bd0 = umma_desc_sw128(smem_addr(wpv));
      for (int gi = 0; gi < ngroups; ++gi) {
        const int a = max(misc->gpad[gi], ps0), z = min(misc->gpad[gi + 1], ps0 + pn);
        const uint32_t tcol = tmem_base + (uint32_t)(gi * nch) * 16u;
        // K steps go round-robin to nch independent accumulators. Descriptor
        // start addresses are in 16-byte units: a K step is 4096 B of rows;
        // 32 B of weights within a 64-slot block, 2048 B per block.
        int ks = (a - misc->gpad[gi]) >> 4, c = ks % nch;
        for (int ps = a - ps0; ps < z - ps0; ps += 16, ++ks) {
          const uint64_t ad = ad0 + (uint64_t)(ps * 16);
          const uint64_t bd = bd0 + (uint64_t)((ps >> 6) * 128 + ((ps & 63) >> 4) * 2);
          umma_f16(tcol + (uint32_t)c * 16u, ad, bd, kIdesc, ks < nch ? 0u : 1u);
          c = (c + 1 == nch) ? 0 : c + 1;
        }
      }
      umma_commit(&misc->pvbar);
      if (ps0 == 0) trace_col(p, 80 + 14, clock64());
    }
    // weight sums of the pass: the 8-slot partials of each (group, head) in
    // slot order
    for (int t = threadIdx.x; t < ngroups * 8; t += kThreads) {
      const int gi = t >> 3, hh = t & 7;
      if (hh < (misc->ghb[gi] >> 16)) {
        const int a = max(misc->gpad[gi], ps0) - ps0, z = min(misc->gpad[gi + 1], ps0 + pn) - ps0;
        auto part = [&](int ps) {
          return *reinterpret_cast<const float*>(wpv + (ps >> 6) * 2048 + 1024 + ((ps & 63) >> 3) * 32 + hh * 4);
        };
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;  // independent chains, combined in a fixed order
        int ps = a;
        for (; ps + 24 < z; ps += 32) {
          s0 += part(ps);
          s1 += part(ps + 8);
          s2 += part(ps + 16);
          s3 += part(ps + 24);
        }
        for (; ps < z; ps += 8) s0 += part(ps);
        misc->lacc[t] += (s0 + s1) + (s2 + s3);
      }
    }
    if (ps0 == 0) trace_sub(p, 12);
    mbar_wait(&misc->pvbar, pvph, p.status);  // the pass's rows and weights may now be overwritten
    if (ps0 == 0) trace_sub(p, 13);
    pvph ^= 1u;
    tc_fence_after();
  }
  if (tr) trace_stamp(p, 13);
  // accumulators -> slots: warp w reads TMEM lanes 32 (w % 4) .. + 31 (d),
  // warps 0-3 the even gather groups, 4-7 the odd ones
  {
    const int q = warp & 3;
    const int d = q * 32 + lane;
    for (int gi = warp >> 2; gi < ngroups; gi += 2) {
      const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
      // accumulators that received at least one K step
      const int used = min(nch, (misc->gpad[gi + 1] - misc->gpad[gi]) >> 4);
      float o[8];
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) o[hh] = 0.f;
      for (int c = 0; c < used; ++c) {  // fixed order: run-to-run identical sums
        uint32_t r[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)((gi * nch + c) * 16), r);
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) o[hh] += __uint_as_float(r[hh]);
      }
#pragma unroll
      for (int hh = 0; hh < 8; ++hh)
        if (hh < nh) slot_put<SHD>(slot_at<SHD>(p, g, j, hb + hh, kSlotO + d), tag, __float_as_uint(o[hh]));
    }
    tc_fence_before();
  }
  for (int t = threadIdx.x; t < ngroups * 8; t += kThreads) {
    const int gi = t >> 3, hh = t & 7;
    if (hh < (misc->ghb[gi] >> 16))
      slot_put<SHD>(slot_at<SHD>(p, g, j, (misc->ghb[gi] & 0xFFFF) + hh, kSlotL), tag, __float_as_uint(misc->lacc[t]));
  }
  for (int hl = threadIdx.x; hl < G; hl += kThreads)
    slot_put<SHD>(slot_at<SHD>(p, g, j, hl, kSlotM), tag, __float_as_uint(MODE == MODE_CALIBRATE ? 0.f : misc->aux[hl]));
  if (tr) trace_stamp(p, 14);
}

// ---------------------------------------------------------------------------
// Dense P.V with the value rows streamed by TMA (16-bit types, head_dim 128,
// contiguous caches; attention.py:64-85). The chunk's value rows of each
// gather group's value head flow through the key ring in 128-row tiles: two
// 64-column boxes with the 128-B swizzle are the MN-major A operand as TMA
// lays them out (8-row atoms 1024 B apart, the second half of head_dim 16 KB
// on). The 4 epilogue warps write each tile's weights exp(l - chunk max),
// rounded to the value type, as the K-major B operand of that ring stage
// (16 head slots, the group's heads and zeros), keep the sums of the rounded
// weights, and arrive on the stage's wfull barrier; warp 0 refills stages
// once their MMAs are done, and one elected thread of warp 1 issues the MMAs
// (M = 128 head_dim rows, N = 16 head slots, K = 16 positions) into the
// group's round-robin TMEM accumulators. The ring state carries on from the
// scorer, so the stages and their barriers serve both phases.
// ---------------------------------------------------------------------------
template <typename T, int D, bool SHD>
__device__ void dense_stream_pv(const DecodeParams& p, int g, int j, int b, int p0, int n,
                                const T* __restrict__ sc, uint8_t* __restrict__ ring, uint8_t* __restrict__ wpv,
                                float* __restrict__ part, Misc* misc, Ring& rg, uint32_t tmem_base, uint32_t& pvph) {
  static_assert(D == 128, "the streamed P.V covers head_dim 128");
  constexpr uint32_t TILE_BYTES = 128u * D * 2u;
  constexpr uint32_t W_BYTES = 4096u;  // weights of one tile: 2 blocks of 64 positions x 16 head slots
  constexpr uint32_t kIdesc = umma_idesc_f16(Num<T>::kDType == SAGA_BF16 ? 1u : 0u, 128, 16) | kUmmaAMajorMN;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NS = p.ns, SH = p.sh, G = p.G;
  const int ngroups = misc->ngroups;
  const int ntl = (n + 127) / 128;
  const int nsteps = ngroups * ntl;
  const int nch = min(4, p.tmem_cols / (16 * max(ngroups, 1)));
  const uint32_t tag = misc->tag;
  if (warp == 1 && lane == 0) {
    misc->vs0 = rg.ms;
    misc->vph0 = rg.mph;
  }
  __syncthreads();
  const uint32_t vs0 = misc->vs0, vph0 = misc->vph0;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int k = 0; k < nsteps && !misc->abort; ++k) {
        if (!mbar_wait(&misc->empty[rg.ps], rg.pph ^ 1u, p.status)) {
          misc->abort = 1;
          break;
        }
        const int gi = k / ntl, t = k - gi * ntl;
        mbar_arrive_expect_tx(&misc->full[rg.ps], TILE_BYTES);
        uint8_t* dst = ring + rg.ps * TILE_BYTES;
#pragma unroll
        for (int kb = 0; kb < D / 64; ++kb)
          tma_load_4d(dst + kb * 16384, &p.vmap, kb * 64, p0 + t * 128, misc->gvh[gi], b, &misc->full[rg.ps]);
        ++issued;
        if (++rg.ps == (uint32_t)NS) {
          rg.ps = 0;
          rg.pph ^= 1u;
        }
      }
      if (misc->abort) {  // drain: the last issued tiles may still be landing
        uint32_t s2 = rg.ps, ph = rg.pph;
        for (int k = 0; k < min(issued, NS); ++k) {
          if (s2 == 0) {
            s2 = NS - 1;
            ph ^= 1u;
          } else {
            --s2;
          }
          mbar_wait(&misc->full[s2], ph, p.status);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int ks = 0, acc_c = 0;  // K steps of the current group; its next accumulator
      for (int k = 0; k < nsteps && !misc->abort; ++k) {
        const int gi = k / ntl, t = k - gi * ntl;
        if (t == 0) ks = acc_c = 0;
        if (!mbar_wait(&misc->full[rg.ms], rg.mph, p.status) ||
            !mbar_wait(&misc->wfull[rg.ms], (rg.wpar >> rg.ms) & 1u, p.status)) {
          misc->abort = 1;
          break;
        }
        rg.wpar ^= 1u << rg.ms;
        tc_fence_after();
        const uint64_t ad0 = umma_desc_mn_sw128(smem_addr(ring + rg.ms * TILE_BYTES), 16384, 1024);
        const uint64_t bd0 = umma_desc_sw128(smem_addr(wpv + rg.ms * W_BYTES));
        const int steps = min(8, (n - t * 128 + 15) >> 4);  // 16-row K steps with real rows
        // The issuing warp shares its scheduler with a weight-building warp,
        // so the loop is kept to a few instructions per MMA: descriptors by
        // constant offsets (16-byte units: 16 rows are 2048 B of A; 32 B of
        // weights within a 64-position block, 2048 B per block), the
        // accumulator by a wrapping counter.
        const uint32_t tg = tmem_base + (uint32_t)(gi * nch) * 16u;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q < steps) {
            umma_f16(tg + (uint32_t)acc_c * 16u, ad0 + (uint64_t)(q * 128),
                     bd0 + (uint64_t)((q >> 2) * 128 + (q & 3) * 2), kIdesc, ks < nch ? 0u : 1u);
            ++ks;
            acc_c = (acc_c + 1 == nch) ? 0 : acc_c + 1;
          }
        }
        umma_commit(&misc->empty[rg.ms]);
        if (++rg.ms == (uint32_t)NS) {
          rg.ms = 0;
          rg.mph ^= 1u;
        }
      }
      umma_commit(&misc->pvbar);  // every MMA of the item, also after an abort
    }
  } else if (warp >= 4 && warp < 8) {
    const int tid = threadIdx.x - 128;  // position within a tile
    float ls[8];
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) ls[hh] = 0.f;
    float stab[16];  // the group's stabilisers; 0 for a head the mask covers whole in this chunk
    for (int k = 0; k < nsteps; ++k) {
      const int gi = k / ntl, t = k - gi * ntl;
      const uint32_t u = vs0 + (uint32_t)k;
      const uint32_t s2 = u % (uint32_t)NS;
      const uint32_t ph = vph0 ^ ((u / (uint32_t)NS) & 1u);
      // the stage's previous MMAs (they read its weights) are complete
      if (!mbar_wait(&misc->empty[s2], ph ^ 1u, p.status)) {
        misc->abort = 1;
        break;
      }
      const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
      if (t == 0) {
#pragma unroll
        for (int hh = 0; hh < 16; ++hh) {
          const float a = hh < nh ? misc->aux[hb + hh] : 0.f;
          stab[hh] = a == -INFINITY ? 0.f : a;
        }
      }
      const int pos = t * 128 + tid;
      uint8_t* wb = wpv + s2 * W_BYTES;
#pragma unroll
      for (int hh = 0; hh < 16; ++hh) {
        T e = Num<T>::from_f(0.f);
        if (hh < nh && pos < n) e = Num<T>::from_f(__expf(Num<T>::to_f(sc[pos * SH + hb + hh]) - stab[hh]));
        *reinterpret_cast<T*>(wb + pv_w_off(tid, hh)) = e;
        if (hh < 8) ls[hh] += Num<T>::to_f(e);  // the rounded weight the MMA multiplies
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->wfull[s2]);
      if (t == ntl - 1) {  // the group's weight sums: per warp, in a fixed order
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) {
          const float v = warp_sum(ls[hh]);
          if (lane == 0) part[((warp - 4) * ngroups + gi) * 8 + hh] = v;
          ls[hh] = 0.f;
        }
      }
    }
  }
  __syncthreads();
  trace_stamp(p, 12);
  mbar_wait(&misc->pvbar, pvph, p.status);
  pvph ^= 1u;
  tc_fence_after();
  trace_stamp(p, 13);
  for (int t2 = threadIdx.x; t2 < ngroups * 8; t2 += kThreads) {
    const int gi = t2 >> 3, hh = t2 & 7;
    misc->lacc[t2] = ((part[(0 * ngroups + gi) * 8 + hh] + part[(1 * ngroups + gi) * 8 + hh]) +
                      part[(2 * ngroups + gi) * 8 + hh]) + part[(3 * ngroups + gi) * 8 + hh];
  }
  // accumulators -> slots: warp w reads TMEM lanes 32 (w % 4) .. + 31 (d),
  // warps 0-3 the even gather groups, 4-7 the odd ones
  {
    const int q = warp & 3;
    const int d = q * 32 + lane;
    const int used = min(nch, (n + 15) / 16);  // accumulators that received a K step
    for (int gi = warp >> 2; gi < ngroups && warp < 8; gi += 2) {
      const int hb = misc->ghb[gi] & 0xFFFF, nh = misc->ghb[gi] >> 16;
      float o[8];
#pragma unroll
      for (int hh = 0; hh < 8; ++hh) o[hh] = 0.f;
      for (int c = 0; c < used; ++c) {  // fixed order: run-to-run identical sums
        uint32_t r[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)((gi * nch + c) * 16), r);
#pragma unroll
        for (int hh = 0; hh < 8; ++hh) o[hh] += __uint_as_float(r[hh]);
      }
#pragma unroll
      for (int hh = 0; hh < 8; ++hh)
        if (hh < nh) slot_put<SHD>(slot_at<SHD>(p, g, j, hb + hh, kSlotO + d), tag, __float_as_uint(o[hh]));
    }
    tc_fence_before();
  }
  __syncthreads();
  for (int t2 = threadIdx.x; t2 < ngroups * 8; t2 += kThreads) {
    const int gi = t2 >> 3, hh = t2 & 7;
    if (hh < (misc->ghb[gi] >> 16))
      slot_put<SHD>(slot_at<SHD>(p, g, j, (misc->ghb[gi] & 0xFFFF) + hh, kSlotL), tag, __float_as_uint(misc->lacc[t2]));
  }
  for (int hl = threadIdx.x; hl < G; hl += kThreads)
    slot_put<SHD>(slot_at<SHD>(p, g, j, hl, kSlotM), tag, __float_as_uint(misc->aux[hl]));
  trace_stamp(p, 14);
}

template <typename T, int D, int MODE, bool SHD, bool PG>
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
  const bool tr = kTrace && p.trace && threadIdx.x == 0 && blockIdx.x < 1024;
  if (tr) trace_col(p, 127, total);
  if (one_batch && total > 0) {
    weights(0, total);
    cp_async_wait<0>();
    __syncthreads();
  }
  if (tr) trace_stamp(p, 12);

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
        issue_rows<T, D, PG>(p, b, p0, list, e0, rows, work, misc);
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
    if (tr && gi == 0) trace_stamp(p, 13);
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
        slot_put<SHD>(slot_at<SHD>(p, g, j, hb + hh, d < D ? kSlotO + d : kSlotL), tag, __float_as_uint(s));
      }
      __syncthreads();
    }
  }
  for (int hl = threadIdx.x; hl < G; hl += kThreads)
    slot_put<SHD>(slot_at<SHD>(p, g, j, hl, kSlotM), tag, __float_as_uint(MODE == MODE_CALIBRATE ? 0.f : misc->aux[hl]));
  if (tr) trace_stamp(p, 14);
}

// ---------------------------------------------------------------------------
// Merge of the group's partials: chunk j produces outputs [lo, hi) of the
// flattened (local head, d) space. All the partials it needs are fetched in
// one burst; sums run in chunk order.
// ---------------------------------------------------------------------------
// One merge level for outputs [lo, lo + nout) (heads hl0 .. hl0 + nhs - 1):
// from nsrc partials, each a slot record at rec(k) (m, l per head; o per
// output), misc->lsum[hh] = l and misc->aux2[hh] = m of the combination, and
// emit(k, o, hh) for every output with o relative to that m. The
// combination order is fixed. A record's partial outputs are [head][d], so
// the slice of source k is one run of consecutive slots from
// rec(k) + kSlotO * G + lo.
template <int D, int MODE, bool SHD, int NT = kThreads, typename Rec, typename Emit>
__device__ void merge_level(const DecodeParams& p, int nsrc, Rec rec, int lo, int nout, int hl0, int nhs, uint32_t tag,
                            uint8_t* scratch, Emit emit, Misc* misc, bool final_level) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t* ml = reinterpret_cast<uint32_t*>(scratch);  // [nhs][nsrc][2]
  uint32_t* ov = ml + nhs * nsrc * 2;                   // [nsrc][nout]
  const int n_ml = nhs * nsrc * 2;
  const int G = p.G;
  const FastDiv div2c((uint32_t)(2 * nsrc)), divn((uint32_t)nout);
  slots_gather<SHD, NT>(
      n_ml + nout * nsrc,
      [&](int i) {
        if (i < n_ml) {
          const int hh = (int)div2c.div((uint32_t)i), r = i - hh * 2 * nsrc;
          return rec(r >> 1) + (kSlotM + (r & 1)) * G + hl0 + hh;
        }
        const int k = i - n_ml;
        const int c = (int)divn.div((uint32_t)k);
        return rec(c) + (kSlotO * G + lo + (k - c * nout));
      },
      tag, ml, p.status);
  trace_sub(p, 25);
  __syncthreads();
  trace_sub(p, 26);
  float* scl = reinterpret_cast<float*>(ov + nout * nsrc);  // [nhs][nsrc]
  for (int hh = warp; hh < nhs; hh += NT / 32) {
    float M = -INFINITY;
    for (int c = lane; c < nsrc; c += 32) M = nanmax(M, __uint_as_float(ml[(hh * nsrc + c) * 2]));
    M = warp_nanmax(M);
    float Ls = 0.f;
    for (int c = lane; c < nsrc; c += 32) {
      const float mc = __uint_as_float(ml[(hh * nsrc + c) * 2]);
      // no source of this level has data (every m is -inf): scale 0, not
      // exp(-inf - -inf); a row empty everywhere still ends as 0 / 0
      const float f = (MODE == MODE_CALIBRATE) ? 1.f : (M == -INFINITY ? 0.f : __expf(mc - M));
      scl[hh * nsrc + c] = f;
      Ls += __uint_as_float(ml[(hh * nsrc + c) * 2 + 1]) * f;
    }
    Ls = warp_sum(Ls);
    if (lane == 0) {
      // calibration renormalises by max(sum p, 1e-12) (attention.py:161)
      misc->lsum[hh] = (MODE == MODE_CALIBRATE && final_level) ? fmaxf(Ls, 1e-12f) : Ls;
      misc->aux2[hh] = M;
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < nout; k += NT) {
    const int hh = (lo + k) / D - hl0;
    float a = 0.f;
    for (int c = 0; c < nsrc; ++c) a += __uint_as_float(ov[c * nout + k]) * scl[hh * nsrc + c];
    emit(k, a, hh);
  }
}

// Merge of the group's partials: the CTAs of this device split the outputs;
// CTA jl merges outputs [jl * per, ...) over the chunks. With sequence
// sharding this happens in two levels: first over this device's chunks, whose
// combined partial is published; then over the devices' partials of the same
// slice (CTA jl of every device covers the same outputs). Every device writes
// all outputs.
template <typename T, int D, int MODE, bool SHD, int NT = kThreads>
__device__ void merge_slice(const DecodeParams& p, int g, int jl, int b, int h0, uint8_t* scratch, Misc* misc) {
  const int G = p.G;
  const int tot = G * D;
  const int per = (tot + p.c_local - 1) / p.c_local;
  const int lo = jl * per, hi = min(tot, lo + per);
  if (lo >= hi) return;
  const int hl0 = lo / D, hl1 = (hi - 1) / D;
  const int nhs = hl1 - hl0 + 1;
  const int nout = hi - lo;
  const uint32_t tag = misc->tag;
  const int c0 = SHD ? p.shard * p.c_local : 0;
  // the group's output of this slice, normalised by the combined weight sum
  const auto write_out = [&](int k, float a, int hh) {
    const int o = lo + k;
    T* out = reinterpret_cast<T*>(p.out) + (int64_t)b * p.o_sb + (int64_t)(h0 + o / D) * p.o_sh + o % D;
    *out = Num<T>::from_f(a / misc->lsum[hh]);
  };
  if constexpr (!SHD) {
    merge_level<D, MODE, false, NT>(
        p, p.c_local, [&](int c) { return slot_at<false>(p, g, c, 0, 0); }, lo, nout, hl0, nhs, tag,
        scratch, write_out, misc, true);
    if (threadIdx.x == 0) trace_stamp(p, 15);
  } else {
    // this device's chunks; their combined partial of the slice is published
    const auto publish = [&](int k, float a, int) {
      const int o = lo + k;
      slot_put<true>(shard_slot(p, g, p.shard, o / D, kSlotO + o % D), tag, __float_as_uint(a));
    };
    merge_level<D, MODE, true>(
        p, p.c_local, [&](int c) { return slot_at<true>(p, g, c0 + c, 0, 0); }, lo, nout, hl0, nhs,
        tag, scratch, publish, misc, false);
    for (int hh = threadIdx.x; hh < nhs; hh += kThreads) {
      slot_put<true>(shard_slot(p, g, p.shard, hl0 + hh, kSlotM), tag, __float_as_uint(misc->aux2[hh]));
      slot_put<true>(shard_slot(p, g, p.shard, hl0 + hh, kSlotL), tag, __float_as_uint(misc->lsum[hh]));
    }
    __syncthreads();  // the staging is reused below
    if (threadIdx.x == 0) trace_stamp(p, 15);
    // every device's partial of the same slice
    merge_level<D, MODE, true>(
        p, p.shards, [&](int sh) { return shard_slot(p, g, sh, 0, 0); }, lo, nout, hl0, nhs, tag,
        scratch, write_out, misc, true);
  }
  trace_sub(p, 21);
}

// ---------------------------------------------------------------------------
// Calibration over 16-bit logits with at most 16 heads per key head: a row of
// the scores buffer is then 16 head slots, 32 bytes, read as two 16-byte
// words, and a thread takes one position with all its heads at a time (the
// per-head loops then run independent chains, and the reads are vectors).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void load_row16(const void* sc, int pl, uint32_t (&w)[8]) {
  const uint4* row = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(sc) + (size_t)pl * 32);
  const uint4 u0 = row[0], u1 = row[1];
  w[0] = u0.x; w[1] = u0.y; w[2] = u0.z; w[3] = u0.w;
  w[4] = u1.x; w[5] = u1.y; w[6] = u1.z; w[7] = u1.w;
}
__device__ __forceinline__ uint32_t slot16(const uint32_t (&w)[8], int h) { return (w[h >> 1] >> ((h & 1) * 16)) & 0xFFFFu; }
// Order-preserving key of 16-bit float bits (bf16 and fp16 alike).
__device__ __forceinline__ uint32_t key16(uint32_t raw) { return (raw & 0x8000u) ? (~raw & 0xFFFFu) : (raw | 0x8000u); }
template <typename T>
__device__ __forceinline__ float raw16_to_f(uint32_t raw) {
  if constexpr (Num<T>::kDType == SAGA_BF16) return __uint_as_float(raw << 16);
  else return __half2float(__ushort_as_half((unsigned short)raw));
}
// The probability of a logit rounded to the dtype (attention.py:133), out of
// line: it is the rare path of the selection loop.
template <typename T>
__device__ __noinline__ float calib_prob_exact(float l, float M, float S) {
  return Num<T>::round(__fdiv_rn(expf(__fsub_rn(l, M)), S));
}

// Warp-wide: the first key k in [lo, hi) with pred(k) true, or hi if none,
// for a predicate that is false then true over the range. Each round the 32
// lanes probe evenly spaced keys and the interval shrinks to the gap before
// the first true probe: 16-bit ranges take four or five rounds.
template <typename Pred>
__device__ __forceinline__ uint32_t warp_first_key(uint32_t lo, uint32_t hi, Pred pred) {
  const int lane = threadIdx.x & 31;
  while (lo < hi) {
    const uint32_t step = (hi - lo + 31) / 32;
    const uint32_t pk = lo + (uint32_t)lane * step;
    const bool valid = pk < hi;
    const uint32_t bal = __ballot_sync(0xffffffffu, valid && pred(pk));
    if (bal == 0u) {  // every probe false: the answer lies past the last probe
      lo = lo + (uint32_t)((hi - lo - 1) / step) * step + 1;
    } else {
      const int f = __ffs(bal) - 1;
      if (f == 0) return lo;                  // lo itself is true
      hi = lo + (uint32_t)f * step;           // true
      lo = lo + (uint32_t)(f - 1) * step + 1;  // past the false probe before it
    }
  }
  return hi;
}

// Radix select: warp-parallel search of the bin holding the `want`-th largest
// key among 256 bins (bin 255 = largest) of a histogram in shared memory.
// Returns the bin; *above = count in higher bins. Called by a full warp.
__device__ __forceinline__ int find_bin(const int* hist256, int want, int* above) {
  const int lane = threadIdx.x & 31;
  int c[8];
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[i] = hist256[255 - lane * 8 - i];
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
template <typename T, int D, int MODE, bool TC, bool MASK, bool SHD, bool PG>
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
  int* toff = reinterpret_cast<int*>(smem + p.sm.sel);       // gather task offsets (sel is free by then)
  uint32_t* occ = reinterpret_cast<uint32_t*>(smem + p.sm.eq);  // gather task occupancy
  float* wbuf = reinterpret_cast<float*>(smem + p.sm.wbuf);
  uint8_t* work = smem + p.sm.work;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = p.G, C = p.C, CL = p.CL, SH = p.sh;
  Ring rg;
  uint32_t tmem_base = 0;
  uint32_t pvph = 0;  // phase of misc->pvbar (every thread waits on every pass)
  constexpr bool kTcPv = uses_tc_pv(TC, D) && sizeof(T) == 2;
  uint8_t* wpv = smem + p.sm.wbuf;

  if (threadIdx.x == 0) trace_col(p, 120, (long long)globaltimer_ns());
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMaxStages; ++s) {
      mbar_init(&misc->full[s], 1);
      mbar_init(&misc->empty[s], 1);
    }
    for (int bb = 0; bb < kScoreBufs; ++bb) {
      mbar_init(&misc->tfull[bb], 1);
      mbar_init(&misc->tempty[bb], 4);
    }
    mbar_init(&misc->pvbar, 1);
    for (int s = 0; s < kMaxStages; ++s) mbar_init(&misc->wfull[s], 4);
    misc->abort = 0;
    mbar_fence_init();
  }
  if constexpr (TC) {
    if (warp == 1) tmem_alloc(&misc->tmem_slot, (uint32_t)p.tmem_cols);
    tc_fence_before();
  }
  __syncthreads();
  if constexpr (TC) {
    tc_fence_after();
    tmem_base = misc->tmem_slot;
  }

  if (threadIdx.x == 0) trace_col(p, 121, (long long)globaltimer_ns());
  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    if constexpr (TC) tc_fence_after();  // TMEM reads of the previous item precede this item's MMAs
    // chunk jl of this device = chunk j of the group (shard-major order)
    const int g = item / p.c_local, jl = item % p.c_local, j = p.shard * p.c_local + jl;
    const int b = g / p.Hk, kh = g % p.Hk, h0 = kh * G;
    const int p0 = jl * CL;
    const int n = min(p.nsel - p0, CL);
    const int nw = (n + 31) / 32;
    int* ctrl = p.ctrl + (size_t)g * kCtrlInts;  // this device's counters of the group
    // calibration statistics: this chunk's, and chunk c's of the group (on the
    // device that owns it when the sequence is sharded)
    ChunkStat* st = p.stats ? p.stats + ((size_t)g * p.c_local + jl) * G : nullptr;
    const auto stat = [&](int c, int hl) -> const ChunkStat* {
      const int owner = SHD ? c / p.c_local : 0;
      return p.stats_peer[owner] + ((size_t)g * p.c_local + (c - owner * p.c_local)) * G + hl;
    };
    const int row0 = b * p.Hq + h0;
    const bool tracing = kTrace && p.trace && threadIdx.x == 0 && item == (int)blockIdx.x && blockIdx.x < 1024;
#define SAGA_TRACE(k) \
  if (tracing) trace_stamp(p, (k));
    SAGA_TRACE(0)
    if constexpr (MODE != MODE_LOGITS && !TC) {  // the tensor-core scorer does it in a helper warp
      if (warp == 3) item_prologue<MODE>(p, b, kh, misc);
    }

    // ---- paged caches: the page of each of the chunk's tiles (read by the
    // scorer's TMA and by the value-row gathers after the next barrier)
    if constexpr (PG) {
      int* tpg = tile_pages(p, misc);
      for (int t = threadIdx.x; t < (n + 127) / 128; t += kThreads) tpg[t] = page_of(p, b, p0 + t * 128);
    }

    // ---- fused append of the decode token (StaticLayer.update's index_copy_).
    // Every chunk of the group writes the new key row (the same values) before
    // it reads the cache, because every chunk scores the tail positions; the
    // chunk that owns the position also writes the value rows it gathers.
    int apos = p.append_pos;
    if (p.append_pos_dev) {
      const long long pd = p.append_pos_dev[0];
      apos = (pd >= 0 && pd < p.L) ? (int)pd : -1;
      if (apos < 0 && threadIdx.x == 0 && jl == 0) set_status(p.status, SAGA_STATUS_APPEND_RANGE);
    }
    if (p.k_new && apos >= 0) {
      const int pos = apos;
      const T* src = reinterpret_cast<const T*>(p.k_new) + (int64_t)b * p.kn_sb + (int64_t)kh * p.kn_sh;
      int apg = 0;  // an append goes to a page of its own sequence
      if constexpr (PG) apg = page_of(p, b, pos);
      T* dst = const_cast<T*>(reinterpret_cast<const T*>(p.k)) + cache_row<PG>(p, p.k_sb, p.k_sh, p.k_sl, b, kh, pos, apg);
      for (int d = threadIdx.x; d < D; d += kThreads) dst[d] = src[d];
      if (p.v_new && pos >= p0 && pos < p0 + n) {
        const int vh_lo = h0 / p.Gv, vh_hi = (h0 + G - 1) / p.Gv;
        for (int i = threadIdx.x; i < (vh_hi - vh_lo + 1) * D; i += kThreads) {
          const int vh = vh_lo + i / D, d = i % D;
          const T* vs = reinterpret_cast<const T*>(p.v_new) + (int64_t)b * p.vn_sb + (int64_t)vh * p.vn_sh;
          T* vd = const_cast<T*>(reinterpret_cast<const T*>(p.v)) + cache_row<PG>(p, p.v_sb, p.v_sh, p.v_sl, b, vh, pos, apg);
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
      score_chunk_tc<T, D, MODE, MASK, PG>(p, b, kh, p0, n, pre0, n_pre, sc, tsc, qop, work, misc, rg, tmem_base);
      const int ej2 = (MODE == MODE_AMORTIZED) ? 2 * epilogue_exp_pairs(G) : 0;
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
        score_range_simt<T, D, MASK, PG>(p, b, kh, tail_start, p.tail, p0, true, qf, sc, work, misc);
      score_range_simt<T, D, MASK, PG>(p, b, kh, p0, n, p0, false, qf, sc, work, misc);
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
        slot_put<SHD>(slot_at<SHD>(p, g, j, hl, kSlotS), tag, __float_as_uint(misc->s[hl]));
      // slot (chunk c, head hl) sits at index c * G + hl of the group's slots
      slots_gather_field<SHD>(p, g, kSlotS, tag, xbuf);
      __syncthreads();
      SAGA_TRACE(2)
      // logit threshold t = m + log(max(thr, 1e-30) * s)  (attention.py:147)
      if constexpr (SHD) {
        // this device's sum, published once; the group's sum over devices
        for (int hl = threadIdx.x; hl < G; hl += kThreads) {
          float s = 0.f;
          for (int c = 0; c < p.c_local; ++c) s += __uint_as_float(xbuf[c * G + hl]);
          if (jl == 0) slot_put<SHD>(shard_slot(p, g, p.shard, hl, kSlotS), tag, __float_as_uint(s));
        }
        __syncthreads();
        slots_gather_shards(p, g, kSlotS, tag, xbuf);
        __syncthreads();
      }
      const int nsum = SHD ? p.shards : p.c_local;  // partial sums in xbuf
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        float s = 0.f;
        for (int c = 0; c < nsum; ++c) s += __uint_as_float(xbuf[c * G + hl]);
        s = Num<T>::round(s);
        const float thr = clamp_min_keep_nan(misc->thr[hl], 1e-30f);
        const float t = __fadd_rn(misc->m[hl], logf(__fmul_rn(thr, s)));
        misc->t[hl] = t;
        if (jl == 0) {  // this device's first chunk (every shard writes its own outputs)
          if (p.logit_thr_out) p.logit_thr_out[row0 + hl] = t;
          if (!isfinite(t)) set_status(p.status, SAGA_STATUS_NONFINITE_THR);
        }
      }
      __syncthreads();
      SAGA_TRACE(8)
      // strict selection x > t (triton_atopn.py:42): per position, the mask of
      // the heads it passes for (zero past n up to the word end), and per-head
      // counts.
      select_heads<T>(sc, SH, G, n, nw, misc, hmask);
      __syncthreads();
      SAGA_TRACE(9)
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        int cnt = 0;
#pragma unroll
        for (int wp = 0; wp < kWarps; ++wp) cnt += misc->cntw[wp][hl];
        misc->i2[hl] = cnt;
        slot_put<SHD>(slot_at<SHD>(p, g, j, hl, kSlotCnt), tag, (uint32_t)cnt);
      }
      // lists, value-row copies and the first pass's weights go out while the
      // counts are exchanged
      gather_begin<T, D, MODE, kTcPv, PG>(p, b, p0, n, sc, hmask, list, toff, occ, work, wpv, misc);
      SAGA_TRACE(3)
      slots_gather_field<SHD>(p, g, kSlotCnt, tag, xbuf);
      __syncthreads();
      SAGA_TRACE(4)
      // exclusive prefix in chunk order: keep the K lowest passing positions
      if constexpr (SHD) {
        // this device's chunks: prefix below chunk jl and total (kept in
        // misc->i3); the total is published once; the earlier devices'
        // totals and the group's total come from the other devices
        for (int hl = threadIdx.x; hl < G; hl += kThreads) {
          int pre = 0, tot = 0;
          for (int c = 0; c < p.c_local; ++c) {
            const int cc = (int)xbuf[c * G + hl];
            if (c < jl) pre += cc;
            tot += cc;
          }
          misc->i3[hl] = pre;
          if (jl == 0) slot_put<SHD>(shard_slot(p, g, p.shard, hl, kSlotCnt), tag, (uint32_t)tot);
        }
        __syncthreads();
        slots_gather_shards(p, g, kSlotCnt, tag, xbuf);
        __syncthreads();
      }
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        int pre = 0, tot = 0;
        if constexpr (SHD) {
          pre = misc->i3[hl];
          for (int sh = 0; sh < p.shards; ++sh) {
            const int cc = (int)xbuf[sh * G + hl];
            if (sh < p.shard) pre += cc;
            tot += cc;
          }
        } else {
          for (int c = 0; c < C; ++c) {
            const int cc = (int)xbuf[c * G + hl];
            if (c < j) pre += cc;
            tot += cc;
          }
        }
        const int mine = misc->i2[hl];
        pre = max(0, pre);  // bounds every offset below even if the slots were corrupt
        misc->i0[hl] = pre;
        misc->i1[hl] = max(0, min(mine, p.buf_k - pre));
        if (jl == 0) {
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
            if (on && k < lim) dst[k] = p.pos_offset + p0 + i;
            o += __popc(bal);
          }
        }
      }
      SAGA_TRACE(11)
      if constexpr (kTcPv) {
        // heads capped at K changed their bits and stabiliser: redo their weights
        pv_weights<T, MODE>(p, sc, hmask, list, wpv, misc, misc->ngroups, 0,
                            min(misc->gpad[misc->ngroups], p.sm.brw), true);
        gather_end_tc<T, D, MODE, SHD, PG>(p, g, j, b, p0, sc, hmask, list, work, wpv, misc, tmem_base, pvph, true);
      }
      else
        gather_end<T, D, MODE, SHD, PG>(p, g, j, b, h0, p0, n, sc, hmask, list, work, wbuf, misc);
    } else if constexpr (MODE == MODE_CALIBRATE) {
      constexpr int KB = Num<T>::kKeyBits;
      constexpr int PASSES = KB / 8;
      const int nsel = p.buf_k;  // min(N, L)
      // [G][HS]: a row stride of 257 words puts the same bin of
      // different heads in different banks (the heads' logits share their
      // busiest bins, and neighbouring lanes hold different heads)
      constexpr int HS = 257;
      int* hsm = reinterpret_cast<int*>(work);
      const bool fast16 = Num<T>::kLowp && SH == 16 && n > 0;
      // the group's histograms [pass][G][256] (shard 0's with sequence sharding)
      int* gh = p.hist_home + (size_t)g * 4 * G * 256;
      int* bctrl = SHD ? p.ctrl_home + (size_t)g * kCtrlInts : ctrl;  // barrier counters
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        st[hl].mx = misc->aux[hl];
        misc->i0[hl] = nsel;  // rank wanted within the current key prefix
        misc->i1[hl] = 0;     // key prefix so far
      }
      int sync_id = 2;
      for (int pass = 0; pass < PASSES; ++pass) {
        const int shift = KB - 8 * (pass + 1);
        for (int i = threadIdx.x; i < G * HS; i += kThreads) hsm[i] = 0;
        __syncthreads();
        if (fast16) {
          // pass 0 also sums exp(l - chunk max) per head (the fast
          // exponential: the threshold is the sum's quotient rounded to the
          // dtype, far coarser than its few-ulp error); the chunks' sums are
          // rescaled to the row max after the exchange
          uint32_t pre[16];
          float cm[16], sacc[16];
#pragma unroll
          for (int h = 0; h < 16; ++h) {
            pre[h] = (pass > 0 && h < G) ? (uint32_t)misc->i1[h] : 0u;
            cm[h] = h < G ? misc->aux[h] : 0.f;
            sacc[h] = 0.f;
          }
          // the two passes as separate loops, each with only its own work
          if (pass == 0) {
            for (int pl0 = threadIdx.x; pl0 < n; pl0 += 2 * kThreads) {
              uint32_t w[2][8];
#pragma unroll
              for (int r = 0; r < 2; ++r) load_row16(sc, min(pl0 + r * kThreads, n - 1), w[r]);
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                if (pl0 + r * kThreads < n) {
#pragma unroll
                  for (int h = 0; h < 16; ++h) {
                    if (h < G) {
                      const uint32_t raw = slot16(w[r], h);
                      atomicAdd(&hsm[h * HS + (key16(raw) >> 8)], 1);
                      sacc[h] += __expf(__fsub_rn(raw16_to_f<T>(raw), cm[h]));
                    }
                  }
                }
              }
            }
          } else {
            for (int pl0 = threadIdx.x; pl0 < n; pl0 += 2 * kThreads) {
              uint32_t w[2][8];
#pragma unroll
              for (int r = 0; r < 2; ++r) load_row16(sc, min(pl0 + r * kThreads, n - 1), w[r]);
#pragma unroll
              for (int r = 0; r < 2; ++r) {
                if (pl0 + r * kThreads < n) {
#pragma unroll
                  for (int h = 0; h < 16; ++h) {
                    const uint32_t key = key16(slot16(w[r], h));
                    if (h < G && (key >> 8) == pre[h]) atomicAdd(&hsm[h * HS + (key & 255u)], 1);
                  }
                }
              }
            }
          }
          if (pass == 0) {
            float* part = reinterpret_cast<float*>(&misc->cntw[0][0]);  // [kWarps][kMaxG]
            const float v = warp_reduce16(sacc, [](float x, float y) { return x + y; });
            if ((lane & 1) == 0 && (lane >> 1) < G) part[warp * kMaxG + (lane >> 1)] = v;
            __syncthreads();
            for (int hl = threadIdx.x; hl < G; hl += kThreads) {
              float v2 = 0.f;
#pragma unroll
              for (int k = 0; k < kWarps; ++k) v2 += part[k * kMaxG + hl];
              st[hl].s = misc->aux[hl] == -INFINITY ? 0.f : v2;  // a fully masked chunk adds nothing
            }
          }
        } else {
          // the chunk's (position, head) pairs in the order i = pl * G + hl,
          // walked with stride kThreads; (pl, hl) advance without a division.
          // Neighbouring lanes hold different heads, so their atomics mostly
          // hit different histograms.
          const int dpl = kThreads / G, dhl = kThreads - dpl * G;
          int pl = threadIdx.x / G, hl = threadIdx.x - (threadIdx.x / G) * G;
          while (pl < n) {
            const uint32_t key = Num<T>::key(Num<T>::to_f(sc[pl * SH + hl]));
            const bool match = (pass == 0) || ((key >> (shift + 8)) == (uint32_t)misc->i1[hl]);
            if (match) atomicAdd(&hsm[hl * HS + ((key >> shift) & 255u)], 1);
            pl += dpl;
            hl += dhl;
            if (hl >= G) {
              hl -= G;
              ++pl;
            }
          }
        }
        __syncthreads();
        trace_sub(p, pass ? 19 : 15);
        for (int i = threadIdx.x; i < G * 256; i += kThreads) {
          const int v = hsm[(i >> 8) * HS + (i & 255)];
          if (v) {
            if constexpr (SHD) atomicAdd_system(&gh[(size_t)pass * G * 256 + i], v);
            else atomicAdd(&gh[(size_t)pass * G * 256 + i], v);
          }
        }
        if (pass == 1 && !fast16) {
          // exp-sum with the global max (attention.py:131-133 softmax)
          for (int hl = warp; hl < G; hl += kWarps) {
            const float M = misc->m[hl];
            float s = 0.f;
            // 16-bit types: the fast exponential, since the threshold is
            // this sum's quotient rounded to the dtype, far coarser than its
            // few-ulp error; fp32 keeps the accurate one
            for (int i = lane; i < n; i += 32) {
              const float d = __fsub_rn(Num<T>::to_f(sc[i * SH + hl]), M);
              s += Num<T>::kLowp ? __expf(d) : expf(d);
            }
            s = warp_sum(s);
            if (lane == 0) st[hl].s = s;
          }
        }
        trace_sub(p, pass ? 20 : 16);
        if constexpr (SHD) group_barrier_sys(&bctrl[sync_id++], C, p.status, &misc->flag);
        else group_barrier(&bctrl[sync_id++], C, true, p.status, &misc->flag);
        trace_sub(p, pass ? 22 : 17);
        // the chunks' statistics of a head, a lane per chunk (loads in flight
        // together): after pass 0 the row max (and, fast path, the exp-sum
        // with each chunk's sum rescaled from its own max); after pass 1 the
        // exp-sum of the other path
        // the group's histograms of this pass, loaded into registers first so
        // that every load is in flight at once (stored below)
        int hv[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int i = threadIdx.x + k * kThreads;
          hv[k] = i < G * 256 ? __ldcg(&gh[(size_t)pass * G * 256 + i]) : 0;
        }
        if ((pass == 0 || !fast16) && C <= 32) {
          // a lane per chunk, both of a warp's heads at once: one round of loads
          const int h0w = warp, h1w = warp + kWarps;
          const bool has0 = h0w < G, has1 = h1w < G;
          const bool on = lane < C;
          float mx0 = -INFINITY, mx1 = -INFINITY, s0 = 0.f, s1 = 0.f;
          if (on && has0) {
            mx0 = __ldcg(&stat(lane, h0w)->mx);
            s0 = __ldcg(&stat(lane, h0w)->s);
          }
          if (on && has1) {
            mx1 = __ldcg(&stat(lane, h1w)->mx);
            s1 = __ldcg(&stat(lane, h1w)->s);
          }
          float M0 = pass == 0 ? warp_nanmax(mx0) : (has0 ? misc->m[h0w] : 0.f);
          float M1 = pass == 0 ? warp_nanmax(mx1) : (has1 ? misc->m[h1w] : 0.f);
          float a0 = 0.f, a1 = 0.f;
          if (pass == 1) {
            a0 = s0;
            a1 = s1;
          } else if (fast16) {
            a0 = (s0 == 0.f) ? 0.f : s0 * __expf(mx0 - M0);
            a1 = (s1 == 0.f) ? 0.f : s1 * __expf(mx1 - M1);
          }
          a0 = warp_sum(a0);
          a1 = warp_sum(a1);
          if (lane == 0) {
            if (has0) {
              if (pass == 0) misc->m[h0w] = M0;
              if (pass == 1 || fast16) misc->s[h0w] = a0;
            }
            if (has1) {
              if (pass == 0) misc->m[h1w] = M1;
              if (pass == 1 || fast16) misc->s[h1w] = a1;
            }
          }
          for (int hl = warp + 2 * kWarps; hl < G; hl += kWarps) {  // G > 16: the rest one by one
            float M = -INFINITY, sm = 0.f, mc = -INFINITY, sc_ = 0.f;
            if (on) {
              mc = __ldcg(&stat(lane, hl)->mx);
              sc_ = __ldcg(&stat(lane, hl)->s);
            }
            M = pass == 0 ? warp_nanmax(mc) : misc->m[hl];
            if (pass == 1) sm = sc_;
            else if (fast16) sm = (sc_ == 0.f) ? 0.f : sc_ * __expf(mc - M);
            sm = warp_sum(sm);
            if (lane == 0) {
              if (pass == 0) misc->m[hl] = M;
              if (pass == 1 || fast16) misc->s[hl] = sm;
            }
          }
        } else if (pass == 0 || !fast16) {
          for (int hl = warp; hl < G; hl += kWarps) {
            float M = -INFINITY;
            if (pass == 0) {
              for (int c0 = 0; c0 < C; c0 += 32)
                if (c0 + lane < C) M = nanmax(M, __ldcg(&stat(c0 + lane, hl)->mx));
              M = warp_nanmax(M);
            } else {
              M = misc->m[hl];
            }
            float sm = 0.f;
            if (pass == 1 || fast16) {
              for (int c0 = 0; c0 < C; c0 += 32) {
                if (c0 + lane < C) {
                  const float sc_ = __ldcg(&stat(c0 + lane, hl)->s);
                  if (pass == 1) {
                    sm += sc_;
                  } else {
                    const float mc = __ldcg(&stat(c0 + lane, hl)->mx);
                    sm += (sc_ == 0.f) ? 0.f : sc_ * __expf(mc - M);
                  }
                }
              }
              sm = warp_sum(sm);
            }
            if (lane == 0) {
              if (pass == 0) misc->m[hl] = M;
              if (pass == 1 || fast16) misc->s[hl] = sm;
            }
          }
        }
        // the group's histograms of this pass into shared memory, then each
        // head's bin from there
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int i = threadIdx.x + k * kThreads;
          if (i < G * 256) hsm[(i >> 8) * HS + (i & 255)] = hv[k];
        }
        __syncthreads();
        for (int hl = warp; hl < G; hl += kWarps) {
          int above = 0;
          const int bin = find_bin(hsm + hl * HS, misc->i0[hl], &above);
          if (lane == 0) {
            misc->i0[hl] -= above;
            misc->i1[hl] = (int)(((uint32_t)misc->i1[hl] << 8) | (uint32_t)bin);
          }
        }
        __syncthreads();
        trace_sub(p, pass ? 23 : 18);
      }
      // the N-th largest logit; its probability is the threshold
      // (attention.py:181-187); softmax output exp(l - M) / S rounded.
      for (int hl = threadIdx.x; hl < G; hl += kThreads) {
        const float lN = Num<T>::unkey((uint32_t)misc->i1[hl]);
        const float pN = Num<T>::round(__fdiv_rn(expf(__fsub_rn(lN, misc->m[hl])), misc->s[hl]));
        misc->t[hl] = lN;
        misc->aux[hl] = pN;
        if (jl == 0 && p.thr_out) p.thr_out[row0 + hl] = pN;  // every device's own table
      }
      __syncthreads();
      // 16-bit logits, at most 16 heads and finite statistics: selection by
      // logit thresholds (below); otherwise per position probabilities.
      bool sel_fast = false;
      if (fast16) {
        int ok = 1;
        for (int hl = threadIdx.x; hl < G; hl += kThreads) {
          const float M = misc->m[hl], S = misc->s[hl], pN = misc->aux[hl];
          if (!(isfinite(M) && isfinite(S) && S > 0.f && pN >= 1e-30f && pN <= 1.f)) ok = 0;
        }
        sel_fast = __syncthreads_and(ok) != 0;
      }
      uint32_t* eqpos = list;  // per position: the heads tied at pN (the lists come later)
      if constexpr (Num<T>::kLowp) if (sel_fast) {
        // Per head, the smallest logits whose probability is > pN and >= pN:
        // a warp search over the dtype's values in key order with the exact
        // probability. The positions then compare their logits with them,
        // two heads per instruction. The probability is non-decreasing in
        // the logit up to expf's few-ulp error, so a position this classifies
        // otherwise than its own probability would has a probability next to
        // pN, a tie that the reference's own rounding could order either way.
        for (int hl = warp; hl < 16; hl += kWarps) {
          float tg = INFINITY, te = INFINITY;  // x > tg passes; x > te passes or ties
          if (hl < G) {
            const float M = misc->m[hl], S = misc->s[hl], pN = misc->aux[hl];
            const auto pgt = [&](uint32_t k) { return calib_prob_exact<T>(Num<T>::unkey(k), M, S) > pN; };
            const auto pge = [&](uint32_t k) { return calib_prob_exact<T>(Num<T>::unkey(k), M, S) >= pN; };
            const uint32_t k0 = Num<T>::key(-INFINITY), k1 = Num<T>::key(INFINITY) + 1u;
            // The N-th largest logit lN has probability pN exactly (the same
            // expression), so the transitions sit just above and at or just
            // below its key: one round of 32 probes on either side finds them
            // unless many neighbouring values share pN; then the full search.
            const uint32_t kN = Num<T>::key(misc->t[hl]);
            uint32_t kg, ke;
            {
              const uint32_t pk = kN + 1u + (uint32_t)lane;
              const uint32_t bal = __ballot_sync(0xffffffffu, pk < k1 && pgt(pk));
              kg = bal ? kN + 1u + (uint32_t)(__ffs(bal) - 1) : warp_first_key(min(kN + 33u, k1), k1, pgt);
            }
            {
              const uint32_t pk = kN - 31u + (uint32_t)lane;  // kN >= k0 >= 127: no wrap
              const uint32_t bal = __ballot_sync(0xffffffffu, pk >= k0 && pge(pk));  // lane 31 (kN) is true
              const int f = __ffs(bal) - 1;
              const uint32_t p0k = kN - 31u;
              ke = f > 0 ? p0k + (uint32_t)f : (p0k > k0 ? warp_first_key(k0, p0k, pge) : k0);
            }
            // prob(-inf) = 0 < pN, so kg, ke > k0 and the values below them exist
            if (kg < k1) tg = Num<T>::unkey(kg - 1u);
            if (ke < k1 && ke > k0) te = Num<T>::unkey(ke - 1u);
          }
          if (lane == 0) {
            misc->t[hl] = tg;
            misc->aux2[hl] = te;
          }
        }
        __syncthreads();
        trace_sub(p, 36);
        using PT = Pair<T>;
        using P = typename PT::P;
        P tg2[8], te2[8];
        uint32_t cg2[8], ce2[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          tg2[k] = PT::pack_rn(misc->t[2 * k], misc->t[2 * k + 1]);
          te2[k] = PT::pack_rn(misc->aux2[2 * k], misc->aux2[2 * k + 1]);
          cg2[k] = ce2[k] = 0u;
        }
        for (int i = threadIdx.x; i < G * (CL / 32); i += kThreads) eqb[i] = 0u;
        __syncthreads();
        for (int i = threadIdx.x; i < nw * 32; i += kThreads) {
          uint32_t gbits = 0, ebits = 0;
          if (i < n) {
            const uint4* row = reinterpret_cast<const uint4*>(sc + (size_t)i * 16);
            const uint4 u0 = row[0], u1 = row[1];
            const P* pa = reinterpret_cast<const P*>(&u0);
            const P* pb = reinterpret_cast<const P*>(&u1);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const P v = k < 4 ? pa[k] : pb[k - 4];
              const uint32_t gm = PT::gt_mask(v, tg2[k]) & 0x00010001u;
              const uint32_t em = PT::gt_mask(v, te2[k]) & ~gm & 0x00010001u;
              cg2[k] += gm;
              ce2[k] += em;
              gbits |= ((gm | (gm >> 15)) & 3u) << (2 * k);
              ebits |= ((em | (em >> 15)) & 3u) << (2 * k);
            }
          }
          hmask[i] = gbits;
          eqpos[i] = ebits;
          // the tied heads also as per-head words, for the trim below (ties
          // are few: one shared-memory OR each)
          while (ebits) {
            const int hl = __ffs(ebits) - 1;
            ebits &= ebits - 1u;
            atomicOr(&eqb[hl * (CL / 32) + (i >> 5)], 1u << (i & 31));
          }
        }
        trace_sub(p, 37);
        trace_sub(p, 38);
        // per-head counts: 16-bit pairs, summed over the warp, then the warps
        int* cnt_w = reinterpret_cast<int*>(work);  // [2][kWarps][16]
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t a = (uint32_t)warp_sum_i((int)cg2[k]), e = (uint32_t)warp_sum_i((int)ce2[k]);
          if (lane == 0) {
            cnt_w[warp * 16 + 2 * k] = (int)(a & 0xFFFFu);
            cnt_w[warp * 16 + 2 * k + 1] = (int)(a >> 16);
            cnt_w[kWarps * 16 + warp * 16 + 2 * k] = (int)(e & 0xFFFFu);
            cnt_w[kWarps * 16 + warp * 16 + 2 * k + 1] = (int)(e >> 16);
          }
        }
        __syncthreads();
        for (int hl = threadIdx.x; hl < G; hl += kThreads) {
          int a = 0, e = 0;
#pragma unroll
          for (int k = 0; k < kWarps; ++k) {
            a += cnt_w[k * 16 + hl];
            e += cnt_w[kWarps * 16 + k * 16 + hl];
          }
          st[hl].cnt = a;
          st[hl].cnt_eq = e;
          misc->i2[hl] = e;
        }
      }
      if (!sel_fast) for (int hl = warp; hl < G; hl += kWarps) {
        const float M = misc->m[hl], S = misc->s[hl], pN = misc->aux[hl];
        // the probability of a logit, rounded to the dtype (attention.py:133)
        const auto prob = [&](float l) { return Num<T>::round(__fdiv_rn(expf(__fsub_rn(l, M)), S)); };
        // 16-bit types: decide "prob > pN" and "prob == pN" from a cheap
        // quotient __expf(l - M) / S where it is clearly away from the edges
        // of pN's rounding interval [lo_b, hi_b], and evaluate prob() exactly
        // near them. __expf's documented error, 2 + 1.173 |x| ulps, stays
        // below 1.3e-5 relative wherever the quotient can reach 1e-31, ten
        // times inside the 1e-4 margin; a tiny pN takes the exact path.
        float lo_b = 0.f, hi_b = 0.f, invS = 0.f;
        bool exact_all = true;
        if constexpr (Num<T>::kLowp) {
          exact_all = !(pN >= 1e-30f && pN <= 1.f && S > 0.f);
          if (!exact_all) {
            const float up = Num<T>::next_up(pN), dn = Num<T>::next_down(pN);
            hi_b = 0.5f * (pN + up);
            lo_b = 0.5f * (pN + dn);
            invS = 1.f / S;
          }
        }
        int cg = 0, ce = 0;
        for (int w = 0; w < nw; ++w) {
          const int i = w * 32 + lane;
          bool gt = false, eq = false;
          if (i < n) {
            const float l = Num<T>::to_f(sc[i * SH + hl]);
            bool exact = exact_all;
            if (!exact) {
              const float qf = __expf(__fsub_rn(l, M)) * invS;
              if (qf != qf || fabsf(qf - hi_b) <= 1e-4f * hi_b || fabsf(qf - lo_b) <= 1e-4f * hi_b) {
                exact = true;
              } else {
                gt = qf > hi_b;
                eq = qf > lo_b && qf < hi_b;
              }
            }
            if (exact) {
              const float pr = prob(l);
              gt = pr > pN;
              eq = pr == pN;
            }
          }
          const uint32_t gb = __ballot_sync(0xffffffffu, gt);
          const uint32_t eb = __ballot_sync(0xffffffffu, eq);
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
      trace_sub(p, 27);
      if constexpr (SHD) group_barrier_sys(&bctrl[sync_id++], C, p.status, &misc->flag);
      else group_barrier(&bctrl[sync_id++], C, true, p.status, &misc->flag);
      trace_sub(p, 28);
      // ties at the N-th probability: the lowest positions fill the set.
      // One warp per head, the chunks' counts loaded a lane each (all in
      // flight together): the total above pN, then in chunk order the ties
      // each chunk keeps, clamp(need - ties before it, 0, its ties), and the
      // rank of this chunk's first kept position.
      for (int hl = warp; hl < G && C <= 32; hl += kWarps) {
        // a lane per chunk, its two counts loaded once
        const int cg = lane < C ? __ldcg(&stat(lane, hl)->cnt) : 0;
        const int ce = lane < C ? __ldcg(&stat(lane, hl)->cnt_eq) : 0;
        const int tot_gt = warp_sum_i(cg);
        const int need = max(0, nsel - tot_gt);
        const int ex = warp_incl_scan(ce) - ce;  // ties of the chunks before this lane's
        const int before = lane < j ? 1 : 0;
        const int pos_pre = warp_sum_i(before * (cg + max(0, min(ce, need - ex))));
        const int eq_pre = warp_sum_i(before * ce);
        if (lane == 0) {
          misc->i2[hl] = max(0, min(misc->i2[hl], need - eq_pre));  // kept ties here
          misc->i3[hl] = max(0, pos_pre);
          if (jl == 0 && p.count_out) p.count_out[row0 + hl] = tot_gt;
        }
      }
      for (int hl = warp; hl < G && C > 32; hl += kWarps) {
        int tot_gt = 0;
        for (int c0 = 0; c0 < C; c0 += 32) {
          const int c = c0 + lane;
          tot_gt += c < C ? __ldcg(&stat(c, hl)->cnt) : 0;
        }
        tot_gt = warp_sum_i(tot_gt);
        const int need = max(0, nsel - tot_gt);
        int eq_pre = 0, pos_pre = 0;  // over the chunks before j
        for (int c0 = 0; c0 < j; c0 += 32) {
          const int c = c0 + lane;
          const int ce = c < j ? __ldcg(&stat(c, hl)->cnt_eq) : 0;
          const int cg = c < j ? __ldcg(&stat(c, hl)->cnt) : 0;
          const int ex = eq_pre + warp_incl_scan(ce) - ce;  // ties of the chunks before c
          pos_pre += warp_sum_i(cg + max(0, min(ce, need - ex)));
          eq_pre += warp_sum_i(ce);
        }
        if (lane == 0) {
          misc->i2[hl] = max(0, min(misc->i2[hl], need - eq_pre));  // kept ties here
          misc->i3[hl] = max(0, pos_pre);
          if (jl == 0 && p.count_out) p.count_out[row0 + hl] = tot_gt;
        }
      }
      __syncthreads();
      trace_sub(p, 29);
      for (int hl = warp; hl < G; hl += kWarps) {
        warp_trim_bits(eqb + hl * (CL / 32), nw, misc->i2[hl]);
        if (!sel_fast) {
          for (int w = lane; w < nw; w += 32) sel[hl * (CL / 32) + w] |= eqb[hl * (CL / 32) + w];
          __syncwarp();
          if (p.sel_idx_out && misc->i3[hl] < p.sel_ld)
            warp_write_positions(sel + hl * (CL / 32), nw, p.pos_offset + p0,
                                 p.sel_idx_out + (size_t)(row0 + hl) * p.sel_ld + misc->i3[hl],
                                 max(0, p.sel_ld - misc->i3[hl]));
        }
      }
      __syncthreads();
      trace_sub(p, 30);
      if (sel_fast) {
        // the kept ties join the passing heads of their positions
        for (int w = warp; w < nw; w += kWarps) {
          const int i = w * 32 + lane;
          if (__ballot_sync(0xffffffffu, eqpos[i] != 0u)) {
            uint32_t add = 0;
            for (int hl = 0; hl < G; ++hl) add |= ((eqb[hl * (CL / 32) + w] >> lane) & 1u) << hl;
            hmask[i] |= add;
          }
        }
        if (p.sel_idx_out) {  // diagnostics: the kept positions from the final masks
          __syncthreads();
          for (int hl = warp; hl < G; hl += kWarps) {
            for (int w = 0; w < nw; ++w) {
              const uint32_t bb = __ballot_sync(0xffffffffu, (hmask[w * 32 + lane] >> hl) & 1u);
              if (lane == 0) sel[hl * (CL / 32) + w] = bb;
            }
            __syncwarp();
            if (misc->i3[hl] < p.sel_ld)
              warp_write_positions(sel + hl * (CL / 32), nw, p.pos_offset + p0,
                                   p.sel_idx_out + (size_t)(row0 + hl) * p.sel_ld + misc->i3[hl],
                                   max(0, p.sel_ld - misc->i3[hl]));
          }
        }
      } else {
        for (int i = threadIdx.x; i < nw * 32; i += kThreads) {
          uint32_t bits = 0;
          if (i < n)
            for (int hl = 0; hl < G; ++hl) bits |= ((sel[hl * (CL / 32) + (i >> 5)] >> (i & 31)) & 1u) << hl;
          hmask[i] = bits;
        }
      }
      __syncthreads();
      trace_sub(p, 34);
      gather_begin<T, D, MODE, kTcPv, PG>(p, b, p0, n, sc, hmask, list, toff, occ, work, wpv, misc);
      if constexpr (kTcPv)
        gather_end_tc<T, D, MODE, SHD, PG>(p, g, j, b, p0, sc, hmask, list, work, wpv, misc, tmem_base, pvph, false);
      else
        gather_end<T, D, MODE, SHD, PG>(p, g, j, b, h0, p0, n, sc, hmask, list, work, wbuf, misc);
    } else {  // MODE_DENSE: misc->aux holds the chunk max from the scoring pass
      bool streamed = false;
      if constexpr (kTcPv && !PG) {
        // value tiles by TMA when the weight buffer holds one tile per ring
        // stage (the layout gives it that for every ring depth it plans)
        if (p.sm.brw >= p.ns * 64) {
          dense_stream_pv<T, D, SHD>(p, g, j, b, p0, n, sc, work, wpv, reinterpret_cast<float*>(list), misc, rg,
                                     tmem_base, pvph);
          streamed = true;
        }
      }
      if (!streamed) {
        gather_begin<T, D, MODE, kTcPv, PG>(p, b, p0, n, sc, hmask, list, toff, occ, work, wpv, misc);
        if constexpr (kTcPv)
          gather_end_tc<T, D, MODE, SHD, PG>(p, g, j, b, p0, sc, hmask, list, work, wpv, misc, tmem_base, pvph, false);
        else
          gather_end<T, D, MODE, SHD, PG>(p, g, j, b, h0, p0, n, sc, hmask, list, work, wbuf, misc);
      }
    }
    __syncthreads();

    // ---- merge of the group's partials, split across its chunks
    trace_sub(p, 24);
    merge_slice<T, D, MODE, SHD>(p, g, jl, b, h0, work, misc);
    SAGA_TRACE(6)

    // ---- the group's last chunk to finish advances the epoch and resets
    // the calibration counters and histograms
    __syncthreads();
    SAGA_TRACE(7)
#undef SAGA_TRACE
    // Completion: the last of this device's chunks of the group resets the
    // counters and advances the epoch. Sharded, that CTA also takes a ticket
    // on shard 0; the last device's ticket advances every device's epoch,
    // and each device's last CTA leaves only after its own epoch advanced.
    // The device's grid stays open until then, so that no device's next
    // launch overwrites slots that a slower device still reads.
    if (threadIdx.x == 0) {
      __threadfence();
      misc->last = (atomicAdd(&ctrl[kCtrlDone], 1) == p.c_local - 1);
    }
    __syncthreads();
    if (misc->last) {
      for (int i = 1 + threadIdx.x; i < kCtrlShardsDone; i += kThreads) ctrl[i] = 0;
      if (MODE == MODE_CALIBRATE) {
        int* gh = p.hist + (size_t)g * 4 * G * 256;
        for (int i = threadIdx.x; i < 4 * G * 256; i += kThreads) gh[i] = 0;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        ctrl[kCtrlDone] = 0;
        if constexpr (!SHD) {
          __threadfence();
          ctrl[0] = (int)tag;  // next launch's tag is tag + 1 (stream-ordered: GPU scope is enough)
        } else {
          int* home = p.ctrl_home + (size_t)g * kCtrlInts;
          __threadfence_system();
          if (atomicAdd_system(&home[kCtrlShardsDone], 1) == p.shards - 1) {
            home[kCtrlShardsDone] = 0;
            __threadfence_system();
            for (int s2 = 0; s2 < p.shards; ++s2)  // every device's epoch
              st_release_sys(p.ctrl_peer[s2] + (size_t)g * kCtrlInts, (int)tag);
          } else {
            unsigned long long t0 = 0;
            for (uint32_t it = 1; ld_acquire_sys(&ctrl[0]) != (int)tag; ++it) {
              __nanosleep(64);
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
          }
        }
      }
    }
    __syncthreads();
  }

  if constexpr (TC) {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, (uint32_t)p.tmem_cols);
    }
  }
  if (threadIdx.x == 0) trace_col(p, 122, (long long)globaltimer_ns());
}


// Kernel entry of one (dtype, head_dim, mode, scorer, mask, sharded, paged) combination.
template <typename T, int D, int MODE, bool TC, bool MASK, bool SHD, bool PG = false>
const void* decode_kernel_ptr() {
  return reinterpret_cast<const void*>(&saga_decode_kernel<T, D, MODE, TC, MASK, SHD, PG>);
}

// Sharded kernels exist for the decode and dense modes on the tensor-core
// path; paged ones (PG) for every mode, not sharded. Paging is a separate
// instantiation so that the contiguous kernels carry none of its code.
template <typename T, bool TC, bool MASK, bool SHD, bool PG = false>
const void* pick_d_mode(int D, int mode) {
  if constexpr (SHD) {
    if (!TC) return nullptr;
    if (D == 64) {
      if (mode == MODE_AMORTIZED) return decode_kernel_ptr<T, 64, MODE_AMORTIZED, TC, MASK, true>();
      if (mode == MODE_CALIBRATE) return decode_kernel_ptr<T, 64, MODE_CALIBRATE, TC, MASK, true>();
      if (mode == MODE_DENSE) return decode_kernel_ptr<T, 64, MODE_DENSE, TC, MASK, true>();
      return nullptr;
    }
    if (mode == MODE_AMORTIZED) return decode_kernel_ptr<T, 128, MODE_AMORTIZED, TC, MASK, true>();
    if (mode == MODE_CALIBRATE) return decode_kernel_ptr<T, 128, MODE_CALIBRATE, TC, MASK, true>();
    if (mode == MODE_DENSE) return decode_kernel_ptr<T, 128, MODE_DENSE, TC, MASK, true>();
    return nullptr;
  } else {
    if (D == 64) {
      switch (mode) {
        case MODE_AMORTIZED: return decode_kernel_ptr<T, 64, MODE_AMORTIZED, TC, MASK, false, PG>();
        case MODE_CALIBRATE: return decode_kernel_ptr<T, 64, MODE_CALIBRATE, TC, MASK, false, PG>();
        case MODE_DENSE: return decode_kernel_ptr<T, 64, MODE_DENSE, TC, MASK, false, PG>();
        default: return decode_kernel_ptr<T, 64, MODE_LOGITS, TC, MASK, false, PG>();
      }
    }
    switch (mode) {
      case MODE_AMORTIZED: return decode_kernel_ptr<T, 128, MODE_AMORTIZED, TC, MASK, false, PG>();
      case MODE_CALIBRATE: return decode_kernel_ptr<T, 128, MODE_CALIBRATE, TC, MASK, false, PG>();
      case MODE_DENSE: return decode_kernel_ptr<T, 128, MODE_DENSE, TC, MASK, false, PG>();
      default: return decode_kernel_ptr<T, 128, MODE_LOGITS, TC, MASK, false, PG>();
    }
  }
}

}  // namespace saga
