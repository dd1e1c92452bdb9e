// Host-side plan and parameters of the fused decode kernel (internal).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "../../include/saga_b200.h"

namespace saga {

enum Mode : int { MODE_AMORTIZED = 0, MODE_CALIBRATE = 1, MODE_DENSE = 2, MODE_LOGITS = 3 };

// Per (group, chunk, local head) statistics published to the other chunks.
struct ChunkStat {
  float mx;     // local max of the logits
  float tmx;    // max over the chunk's part of the tail (amortized)
  float s;      // partial exp-sum
  int cnt;      // passing count (amortized) / greater-than count (calibration)
  int cnt_eq;   // calibration: count equal to the N-th probability
  int pad[3];
};

constexpr int kCtrlInts = 32;   // control counters per group
constexpr int kCtrlDone = 31;   // index of the group's completion counter (this device's chunks)
constexpr int kCtrlShardsDone = 30;  // sharded, on shard 0: devices whose chunks are all done
constexpr int kMaxG = 32;       // query heads per key head supported
constexpr int kMaxStages = 4;   // K-tile ring depth of the tensor-core scorer
constexpr int kScoreBufs = 2;   // TMEM accumulators of the tensor-core scorer (16 columns each)
constexpr int kMaxGatherGroups = 64;
constexpr int kMaxShards = 8;   // devices a sequence can be sharded over

// Shared-memory carve of the fused kernel, in bytes from a 1024-aligned base.
struct SmemLayout {
  int misc, qop, scores, tail, sel, eq, hmask, list, wbuf, work, xbuf, tpg, total;
  int work_bytes;  // K-tile ring / SIMT stages, then V rows, histograms, reductions
  int br;          // value rows per gather batch (CUDA-core P.V)
  int brw;         // value-row slots per pass of the tensor-core P.V (multiple of 16; 0 = not used)
};

// The tensor-core P.V (tcgen05, V rows as the M = head_dim operand) serves
// 16-bit types at head_dim 128 on the tensor-core scorer path.
__host__ __device__ constexpr bool uses_tc_pv(bool tc, int D) { return tc && D == 128; }

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

// G query heads per key head, head dim D, CL positions per chunk, esize bytes
// per element, C chunks per group (all devices' with sequence sharding), of
// which c_local on this device (they split the merged outputs), tensor-core
// scorer with ns stages, nvh value heads per group.
__host__ __device__ inline SmemLayout smem_layout(int G, int D, int CL, int esize, int C, int c_local, bool tc,
                                                 int ns, int nvh) {
  SmemLayout l;
  const int SH = G <= 16 ? 16 : 32;  // head slots per position of the logits
  const int rowb = D * esize;
  int work = tc ? ns * 128 * rowb : 2 * 64 * (rowb + 16);
  const int red = 8 * 8 * D * 4 + 8 * 8 * 4;  // per-warp values and weight sums
  const int hist = G * 257 * 4;  // calibration histograms, rows padded to 257 words
  // merge staging: (m, l) and scale per covered head and chunk, o per output and chunk
  const int per = (G * D + c_local - 1) / c_local;
  const int nhs = per / D + 2;
  const int merge = 4 * (nhs * C * 3 + per * C + per) + 256;
  // per-chunk exchange staging, at the end of the work area: the count
  // exchange runs while value rows are landing at its start
  const int xchg = align_up(4 * C * G, 128);
  work = work > red ? work : red;
  work = work > hist ? work : hist;
  work = work > merge ? work : merge;
  work = work > xchg + 16 * rowb ? work : xchg + 16 * rowb;  // at least one 16-row P.V step
  work = align_up(work, 1024);
  int br = (work - xchg) / rowb;
  br = br > 512 ? 512 : br;
  const bool tcpv = uses_tc_pv(tc, D);
  // 16-row units of 8-row x 256-B swizzle-atom pairs below the exchange staging
  const int brw = tcpv ? ((work - xchg) / (16 * rowb)) * 16 : 0;
  int off = 0;
  l.misc = off;   off += 6144;
  l.qop = off;    off += align_up(tc ? (D / 64) * 2048 : G * D * 4, 1024);
  l.work = off;   off += work;
  l.xbuf = l.work + work - xchg;
  l.scores = off; off += align_up(SH * CL * esize, 128);
  l.sel = off;    off += align_up(G * (CL / 32) * 4, 128);
  l.eq = off;     off += align_up(G * (CL / 32) * 4, 128);
  l.hmask = off;  off += align_up(CL * 4, 128);  // selected heads of each position
  // gather lists; during scoring the same bytes hold the logits of the <= 3 tail tiles
  const int list_b = nvh * CL * 4, tail_b = tc ? 3 * 128 * 16 * esize : 0;
  l.list = off;   off += align_up(list_b > tail_b ? list_b : tail_b, 128);
  l.tail = l.list;
  if (tcpv) {  // bf16/fp16 weights, K-major 128-B swizzle blocks of 16 head slots x 64 rows
    off = align_up(off, 1024);
    l.wbuf = off;  off += align_up((brw + 63) / 64 * 2048, 1024);
  } else {     // fp32 weights [br][8], then the cross-warp reduction buffer
    l.wbuf = off;  off += align_up(br * 8 * 4, 128) + align_up(8 * (D + 1) * 4, 128);
  }
  l.tpg = off;    off += align_up(4 * (CL / 128), 128);  // paged caches: page of each 128-row tile of the chunk
  l.total = off + 1024;  // slack to align the dynamic base to 1024
  l.work_bytes = work;
  l.br = br;
  l.brw = brw;
  return l;
}

struct DecodeParams {
  CUtensorMap tmap;  // key cache, 4-D {D, L, Hk, B}, 64 x 128 boxes, 128-B swizzle (tensor-core path)
  CUtensorMap vmap;  // value cache, the same form over {D, L, Hv, B} (dense mode, tensor-core P.V)
  int B, Hq, Hk, Hv, D, L, G, Gv;
  int C, CL, items, tail, buf_k, ns, nvh, sh;
  int tmem_cols;  // TMEM columns per CTA: the scorer's kScoreBufs x 16, or up to 4 x 16 per gather group for the P.V
  const void* q; int64_t q_sb, q_sh;
  const void* k; int64_t k_sb, k_sh, k_sl;
  const void* v; int64_t v_sb, v_sh, v_sl;
  const void* mask; int mask_dtype; int64_t m_sb, m_sh, m_sl;
  float scaling;
  const float* thr_in; float* thr_out;
  void* out; int64_t o_sb, o_sh;
  const void* k_new; int64_t kn_sb, kn_sh;
  const void* v_new; int64_t vn_sb, vn_sh;
  int append_pos;
  const long long* append_pos_dev;  // when set, the append position is read from here
  // paged caches: pools [num_pages][H][page_len][D], k_sb / v_sb the page strides
  const int* page_table;  // [B][pt_sb] page numbers, or null (contiguous caches)
  long long pt_sb;
  int page_len, page_shift, num_pages;
  float* logit_thr_out; int* count_out; int* sel_idx_out; int sel_ld;
  void* logits_out; int64_t lo_ld;
  int* ctrl; ChunkStat* stats; int* hist;
  unsigned long long* slots;  // [group][chunk][head][D + 4] epoch-tagged exchange slots
  // sequence sharding: chunk c of a group lives on shard c / c_local; its slots
  // are in slot_base[shard] (this device's or a peer's workspace), [group]
  // [c % c_local][head][D + 4]; the epoch and completion counters are shard 0's
  int nsel, pos_offset, shards, shard, c_local;
  unsigned long long* slot_base[kMaxShards];
  int* ctrl_home;               // shard 0's control counters (device tickets, calibration barriers)
  ChunkStat* stats_peer[kMaxShards];  // calibration: every shard's chunk statistics [group][c_local][G]
  int* hist_home;               // calibration: shard 0's histograms (every device adds into them)
  int* ctrl_peer[kMaxShards];   // every shard's control counters (epoch releases)
  int* status;
  long long* trace;
  SmemLayout sm;
};

struct DecodePlan {
  int G, Gv, groups, C, CL, items, grid, smem, ns, nvh, tmem_cols;
  bool cooperative, tc;
  size_t ws_ctrl, ws_stats, ws_part, ws_hist, ws_total;
};

// Builds the plan for `args` and `mode` on the current device.
int make_decode_plan(const SagaAttnArgs* a, int mode, DecodePlan* plan, std::string* err);

// Launches the fused kernel. `args` were validated by the caller.
int launch_decode(const SagaAttnArgs* a, int mode, cudaStream_t stream, std::string* err,
                  std::string* launched);

}  // namespace saga
