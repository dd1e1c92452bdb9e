// Host-side plan and parameters of the fused decode kernel (internal).
#pragma once

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
constexpr int kCtrlDone = 31;   // index of the group's completion counter
constexpr int kMaxG = 32;       // query heads per key head supported

// Shared-memory carve of the fused kernel (bytes from the dynamic base).
struct SmemLayout {
  int misc, q, scores, sel, eq, list, stage, total;
  int stage_bytes;
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int G, int D, int CL, int esize, int C) {
  SmemLayout l;
  int off = 0;
  l.misc = off;   off += 2048;
  l.q = off;      off += align_up(G * D * 4, 128);
  l.scores = off; off += align_up(G * CL * 4, 128);
  l.sel = off;    off += align_up(G * (CL / 32) * 4, 128);
  l.eq = off;     off += align_up(G * (CL / 32) * 4, 128);
  l.list = off;   off += align_up(CL * 4, 128);
  l.stage = off;
  const int pitch = D * esize + 16;
  int st = 2 * 64 * pitch;                         // two staged K sub-tiles
  int red = 8 * 8 * D * 4;                         // gather reduction (8 warps x 8 heads)
  int hist = G * 256 * 4;                          // radix histogram
  int merge = (G + 2 * C + 64) * 4 + 64 * 4;       // merge scale factors (bound)
  st = st > red ? st : red;
  st = st > hist ? st : hist;
  st = st > merge ? st : merge;
  l.stage_bytes = align_up(st, 128);
  off += l.stage_bytes;
  l.total = off;
  return l;
}

struct DecodeParams {
  int B, Hq, Hk, Hv, D, L, G, Gv;
  int C, CL, items, tail, buf_k;
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
  float* logit_thr_out; int* count_out; int* sel_idx_out; int sel_ld;
  void* logits_out; int64_t lo_ld;
  int* ctrl; ChunkStat* stats; float* partials; int* hist;
  int* status;
  SmemLayout sm;
};

struct DecodePlan {
  int G, Gv, groups, C, CL, items, grid, smem;
  bool cooperative;
  size_t ws_ctrl, ws_stats, ws_part, ws_hist, ws_total;
};

// Builds the plan for `args` and `mode` on the current device.
int make_decode_plan(const SagaAttnArgs* a, int mode, DecodePlan* plan, std::string* err);

// Launches the fused kernel. `args` were validated by the caller.
int launch_decode(const SagaAttnArgs* a, int mode, cudaStream_t stream, std::string* err,
                  std::string* launched);

}  // namespace saga
