// Host side of the fused decode kernel: plan (chunking, shared-memory carve,
// grid) and launch. The kernels are instantiated per dtype in decode_bf16.cu,
// decode_fp16.cu and decode_fp32.cu (device code in decode_kernel.cuh).
#include <array>
#include <map>
#include <mutex>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"
#include "decode_internal.h"

namespace saga {

const void* pick_decode_kernel_bf16(int D, int mode, bool tc, bool mask, bool shard, bool paged);
const void* pick_decode_kernel_fp16(int D, int mode, bool tc, bool mask, bool shard, bool paged);
const void* pick_decode_kernel_fp32(int D, int mode, bool tc, bool mask, bool shard, bool paged);

namespace {

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
  int smem_per_sm = 0;
};

DevInfo dev_info() {
  static thread_local int cached_dev = -1;
  static thread_local DevInfo info;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&info.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&info.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cached_dev = dev;
  }
  return info;
}

int esize_of(int dt) { return dt == SAGA_FP32 ? 4 : 2; }

const void* pick_kernel(int dt, int D, int mode, bool tc, bool mask, bool shard, bool paged) {
  if (dt == SAGA_BF16) return pick_decode_kernel_bf16(D, mode, tc, mask, shard, paged);
  if (dt == SAGA_FP16) return pick_decode_kernel_fp16(D, mode, tc, mask, shard, paged);
  return pick_decode_kernel_fp32(D, mode, false, mask, shard, paged);
}

const char* mode_name(int mode) {
  switch (mode) {
    case MODE_AMORTIZED: return "saga_decode_kernel<amortized>";
    case MODE_CALIBRATE: return "saga_decode_kernel<calibrate>";
    case MODE_DENSE: return "saga_decode_kernel<dense>";
    default: return "saga_decode_kernel<logits>";
  }
}

size_t al256(size_t x) { return (x + 255) / 256 * 256; }

// Gather groups of one key-head group: for each value head it touches, one
// group per batch of <= 8 of its query heads. Sizes the position list.
int gather_groups_per_group(int Hq, int Hk, int Hv) {
  const int G = Hq / Hk, Gv = Hq / Hv;
  int m = 1;
  for (int kh = 0; kh < Hk; ++kh) {
    const int h0 = kh * G;
    int ng = 0;
    for (int vh = h0 / Gv; vh <= (h0 + G - 1) / Gv; ++vh) {
      const int nh = std::min(h0 + G, (vh + 1) * Gv) - std::max(h0, vh * Gv);
      ng += (nh + 7) / 8;
    }
    m = std::max(m, ng);
  }
  return m;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace

// The kernel's dynamic shared-memory limit is a per-function, per-device
// attribute; plans of different shapes may share a kernel, so it only rises.
static int raise_smem_limit(const void* kfn, int smem, std::string* err = nullptr) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> set_to;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  int& cur = set_to[{dev, kfn}];
  if (smem <= cur) return 0;
  const cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear it: the caller reports this call's own error
    if (err)
      *err = std::string("cudaFuncSetAttribute(") + std::to_string(smem) + " bytes of shared memory): " +
             cudaGetErrorString(e);
    return -1;
  }
  cur = smem;
  return 0;
}

static int compute_decode_plan(const SagaAttnArgs* a, int mode, DecodePlan* pl, std::string* err);

// Plans depend only on the device and the shapes, so they are computed once:
// a decode step otherwise pays for the occupancy query and the attribute call
// twice (workspace size, then launch).
int make_decode_plan(const SagaAttnArgs* a, int mode, DecodePlan* pl, std::string* err) {
  int dev = 0;
  cudaGetDevice(&dev);
  const std::array<long long, 13> key = {dev, mode, a->dtype, a->B, a->Hq, a->Hk, a->Hv, a->D, a->L, a->nsel,
                                         a->shards, a->mask != nullptr, a->page_table != nullptr};
  static std::mutex mu;
  static std::map<std::array<long long, 13>, DecodePlan> plans;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = plans.find(key);
    if (it != plans.end()) {
      *pl = it->second;
      return SAGA_OK;
    }
  }
  const int rc = compute_decode_plan(a, mode, pl, err);
  if (rc == SAGA_OK) {
    std::lock_guard<std::mutex> lock(mu);
    plans[key] = *pl;
  }
  return rc;
}

static int compute_decode_plan(const SagaAttnArgs* a, int mode, DecodePlan* pl, std::string* err) {
  const DevInfo di = dev_info();
  if (di.sms <= 0) {
    *err = "no CUDA device";
    return SAGA_ERR_CUDA;
  }
  const int G = a->Hq / a->Hk, Gv = a->Hq / a->Hv;
  const int groups = a->B * a->Hk;
  const int nsel = (a->nsel > 0) ? a->nsel : a->L;  // this call's own positions
  const int ntiles = (nsel + kTile - 1) / kTile;
  const int es = esize_of(a->dtype);
  const bool tc = (a->dtype != SAGA_FP32) && G <= 16;
  const int ngg = gather_groups_per_group(a->Hq, a->Hk, a->Hv);  // list rows per position
  // tensor-core path: one CTA per SM, deepest K ring that fits; else two per
  // SM, or one when not even a one-tile chunk fits half an SM's shared memory
  int budget = tc ? di.smem_optin : std::min(di.smem_optin, 113 * 1024);
  // the exchanges stage every chunk of the group: with sequence sharding,
  // the other devices' chunks too
  const int shards = a->shards > 1 ? a->shards : 1;
  const int cbound = std::min(ntiles, 4096) * shards;
  const int target = tc ? di.sms : 2 * di.sms;
  int c_par = std::max(1, target / std::max(1, groups));
  // Deepest K ring whose chunk still lets every group run in one wave; if no
  // ring depth allows that, the deepest one that fits.
  auto tiles_for = [&](int stages) {
    int mt = 0;
    for (int t = 1; t <= ntiles; ++t) {
      if (smem_layout(G, a->D, t * kTile, es, cbound, std::max(1, cbound / shards), tc, stages, ngg).total <= budget) mt = t;
      else break;
    }
    return mt;
  };
  int ns = tc ? kMaxStages : 2, max_tiles = tiles_for(ns);
  if (!tc && max_tiles == 0) {  // one CTA per SM: chunks for one wave of them
    budget = di.smem_optin;
    max_tiles = tiles_for(ns);
    c_par = std::max(1, di.sms / std::max(1, groups));
  }
  if (tc) {
    bool one_wave = false;
    for (int s = kMaxStages; s >= 2; --s) {
      const int mt = tiles_for(s);
      if (mt > 0 && (ntiles + mt - 1) / mt <= c_par) {
        ns = s;
        max_tiles = mt;
        one_wave = true;
        break;
      }
    }
    if (!one_wave) {
      // The items run in rounds of one per SM. Ring depth and chunk length
      // with the fewest rounds x (tiles per chunk + about six tiles' worth of
      // per-item exchanges and merge); deeper rings win ties. E.g. dense
      // decode with unmerged key heads at config 2: 18 chunks of 15 tiles per
      // group on a 3-stage ring run in 2 rounds, not 20 of 13 in 3.
      long best = -1;
      for (int s = kMaxStages; s >= 2; --s) {
        const int mt = tiles_for(s);
        for (int t = mt; t >= 1; --t) {
          const long cc = (ntiles + t - 1) / t;
          const long rounds = ((long)groups * cc + target - 1) / target;
          const long cost = rounds * (t + 6);
          if (best < 0 || cost < best) {
            best = cost;
            ns = s;
            max_tiles = t;
          }
        }
      }
    }
  }
  if (max_tiles == 0) {
    *err = "shapes need more shared memory than one CTA has";
    return SAGA_ERR_UNSUPPORTED;
  }
  const int c_fit = (ntiles + max_tiles - 1) / max_tiles;
  int C = std::max(c_fit, std::min(c_par, ntiles));
  int tiles = (ntiles + C - 1) / C;
  C = (ntiles + tiles - 1) / tiles;
  // The layout is not monotone in C: fewer chunks shrink the exchange staging
  // at the end of the work area, which lends the P.V weight buffer more rows.
  // Re-check the final layout and shorten the chunks until it fits.
  SmemLayout sm = smem_layout(G, a->D, tiles * kTile, es, C * shards, C, tc, ns, ngg);
  while (sm.total > budget && tiles > 1) {
    --tiles;
    C = (ntiles + tiles - 1) / tiles;
    sm = smem_layout(G, a->D, tiles * kTile, es, C * shards, C, tc, ns, ngg);
  }
  if (sm.total > budget) {
    *err = "shapes need more shared memory than one CTA has";
    return SAGA_ERR_UNSUPPORTED;
  }
  const int CL = tiles * kTile;

  pl->G = G;
  pl->Gv = Gv;
  pl->groups = groups;
  pl->C = C;
  pl->CL = CL;
  pl->items = groups * C;
  pl->smem = sm.total;
  pl->ns = ns;
  pl->nvh = ngg;
  pl->tc = tc;
  pl->cooperative = (mode != MODE_LOGITS);
  // TMEM columns per CTA: the scorer's kScoreBufs 16-column accumulators, or
  // up to 4 x 16 columns per gather group for the tensor-core P.V
  pl->tmem_cols = 16 * kScoreBufs;
  if (uses_tc_pv(tc, a->D)) {
    // up to 4 16-column accumulators per gather group, within 256 columns
    const int want = 16 * ngg * std::max(1, std::min(4, 256 / (16 * ngg)));
    while (pl->tmem_cols < want) pl->tmem_cols *= 2;  // ngg <= 16 on this path: at most 256
  }
  const void* kfn = pick_kernel(a->dtype, a->D, mode, tc, a->mask != nullptr, shards > 1, a->page_table != nullptr);
  if (!kfn) {
    *err = "no kernel for this combination of dtype, head_dim, op, sharding and paging";
    return SAGA_ERR_UNSUPPORTED;
  }
  // The CTAs on one SM must fit its 512 TMEM columns together (an allocation
  // that does not fit would wait): ask for enough shared memory that no more
  // of them share an SM.
  const int max_per_sm = tc ? std::max(1, 512 / pl->tmem_cols) : 1 << 30;
  if (tc && di.smem_per_sm > 0) {
    const int floor_smem = di.smem_per_sm / (max_per_sm + 1) + 1024;
    if (pl->smem < floor_smem) pl->smem = std::min(floor_smem, budget);
  }
  if (raise_smem_limit(kfn, pl->smem, err) != 0) return SAGA_ERR_CUDA;
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kfn, kThreads, pl->smem) != cudaSuccess || nb <= 0) {
    *err = "occupancy query failed";
    cudaGetLastError();
    return SAGA_ERR_CUDA;
  }
  if (nb > max_per_sm) {
    *err = "cannot bound the CTAs per SM to the TMEM columns they need";
    return SAGA_ERR_UNSUPPORTED;
  }
  const int cap = nb * di.sms;
  if (pl->cooperative && C > cap) {
    *err = "a group needs more co-resident CTAs than the device holds";
    return SAGA_ERR_UNSUPPORTED;
  }
  pl->grid = pl->cooperative ? std::min(pl->items, cap) : pl->items;

  pl->ws_ctrl = 0;
  pl->ws_hist = al256((size_t)groups * kCtrlInts * 4);
  pl->ws_stats = pl->ws_hist + (mode == MODE_CALIBRATE ? al256((size_t)groups * 4 * G * 256 * 4) : 0);
  pl->ws_part = pl->ws_stats + (mode == MODE_CALIBRATE ? al256((size_t)groups * C * G * sizeof(ChunkStat)) : 0);
  // chunk slots, then (sequence sharding) the device's combined values
  pl->ws_total = pl->ws_part + al256((size_t)groups * C * G * (a->D + 4) * 8) +
                 (shards > 1 ? al256((size_t)groups * G * (a->D + 4) * 8) : 0);
  return SAGA_OK;
}

int launch_decode(const SagaAttnArgs* a, int mode, cudaStream_t stream, std::string* err,
                  std::string* launched) {
  DecodePlan pl;
  int rc = make_decode_plan(a, mode, &pl, err);
  if (rc) return rc;
  if (mode != MODE_LOGITS && (a->workspace == nullptr || a->workspace_bytes < pl.ws_total)) {
    *err = "workspace missing or smaller than saga_workspace_bytes()";
    return SAGA_ERR_WORKSPACE;
  }
  DecodeParams p;
  memset(&p, 0, sizeof(p));
  p.B = a->B; p.Hq = a->Hq; p.Hk = a->Hk; p.Hv = a->Hv; p.D = a->D; p.L = a->L;
  p.G = pl.G; p.Gv = pl.Gv;
  const int shards = a->shards > 1 ? a->shards : 1;
  p.C = pl.C * shards; p.CL = pl.CL; p.items = pl.items; p.ns = pl.ns; p.nvh = pl.nvh;
  p.c_local = pl.C;
  p.shards = shards;
  p.shard = shards > 1 ? a->shard : 0;
  p.nsel = (a->nsel > 0) ? a->nsel : a->L;
  p.pos_offset = a->pos_offset;
  p.sh = pl.G <= 16 ? 16 : 32;
  p.tmem_cols = pl.tmem_cols;
  p.tail = std::min(kTail, a->L);
  if (mode == MODE_AMORTIZED) p.buf_k = std::min(2 * a->top_n, a->L);
  else if (mode == MODE_CALIBRATE) p.buf_k = std::min(a->top_n, a->L);
  else p.buf_k = a->L;
  p.q = a->q; p.q_sb = a->q_sb; p.q_sh = a->q_sh;
  p.k = a->k; p.k_sb = a->k_sb; p.k_sh = a->k_sh; p.k_sl = a->k_sl;
  p.v = a->v; p.v_sb = a->v_sb; p.v_sh = a->v_sh; p.v_sl = a->v_sl;
  p.mask = a->mask; p.mask_dtype = a->mask_dtype; p.m_sb = a->m_sb; p.m_sh = a->m_sh; p.m_sl = a->m_sl;
  p.scaling = a->scaling;
  p.thr_in = a->thr_in; p.thr_out = a->thr_out;
  p.out = a->out; p.o_sb = a->o_sb; p.o_sh = a->o_sh;
  p.k_new = a->k_new; p.kn_sb = a->kn_sb; p.kn_sh = a->kn_sh;
  p.v_new = a->v_new; p.vn_sb = a->vn_sb; p.vn_sh = a->vn_sh;
  p.append_pos = a->append_pos;
  p.append_pos_dev = reinterpret_cast<const long long*>(a->append_pos_dev);
  p.page_table = a->page_table;
  p.pt_sb = a->pt_sb;
  p.page_len = a->page_table ? a->page_len : 0;
  p.page_shift = 0;
  while (p.page_len > 0 && (1 << p.page_shift) < p.page_len) ++p.page_shift;
  p.num_pages = a->page_table ? a->num_pages : 0;
  p.logit_thr_out = a->logit_thr_out; p.count_out = a->count_out;
  p.sel_idx_out = a->sel_idx_out; p.sel_ld = a->sel_ld;
  p.logits_out = a->logits_out; p.lo_ld = a->lo_ld;
  uint8_t* ws = reinterpret_cast<uint8_t*>(a->workspace);
  if (mode != MODE_LOGITS) {
    p.ctrl = reinterpret_cast<int*>(ws + pl.ws_ctrl);
    p.hist = mode == MODE_CALIBRATE ? reinterpret_cast<int*>(ws + pl.ws_hist) : nullptr;
    p.stats = mode == MODE_CALIBRATE ? reinterpret_cast<ChunkStat*>(ws + pl.ws_stats) : nullptr;
    p.slots = reinterpret_cast<unsigned long long*>(ws + pl.ws_part);
    p.ctrl_home = p.ctrl;
    p.slot_base[0] = p.slots;
    p.ctrl_peer[0] = p.ctrl;
    p.stats_peer[0] = p.stats;
    p.hist_home = p.hist;
    if (shards > 1) {  // every shard's workspace has the same layout
      for (int s2 = 0; s2 < shards; ++s2) {
        uint8_t* w = reinterpret_cast<uint8_t*>(a->shard_workspaces[s2]);
        p.slot_base[s2] = reinterpret_cast<unsigned long long*>(w + pl.ws_part);
        p.ctrl_peer[s2] = reinterpret_cast<int*>(w + pl.ws_ctrl);
        if (mode == MODE_CALIBRATE) {
          p.stats_peer[s2] = reinterpret_cast<ChunkStat*>(w + pl.ws_stats);
          if (s2 == 0) p.hist_home = reinterpret_cast<int*>(w + pl.ws_hist);
        }
      }
      p.ctrl_home = p.ctrl_peer[0];
    }
  }
  p.status = a->status;
  p.trace = reinterpret_cast<long long*>(a->trace);
  p.sm = smem_layout(pl.G, a->D, pl.CL, esize_of(a->dtype), pl.C * shards, pl.C, pl.tc, pl.ns, pl.nvh);

  if (pl.tc) {
    auto enc = encode_fn();
    if (!enc) {
      *err = "cuTensorMapEncodeTiled unavailable";
      return SAGA_ERR_CUDA;
    }
    const uint64_t es = 2;
    const bool paged = a->page_table != nullptr;
    // strides of size-1 dims do not matter; keep them valid (multiples of 16 B)
    // contiguous: {D, L, H, B}; paged: {D, page_len, H, num_pages} over the pool
    auto encode = [&](CUtensorMap* out, const void* base, int H, int64_t s_l, int64_t s_h, int64_t s_b,
                      const char* what) -> int {
      const uint64_t rows = paged ? (uint64_t)a->page_len : (uint64_t)a->L;
      const uint64_t outer = paged ? (uint64_t)a->num_pages : (uint64_t)a->B;
      const uint64_t sl = (uint64_t)s_l * es;
      const uint64_t sh = H > 1 ? (uint64_t)s_h * es : sl * rows;
      const uint64_t sb = outer > 1 ? (uint64_t)s_b * es : sh * (uint64_t)H;
      cuuint64_t dims[4] = {(cuuint64_t)a->D, (cuuint64_t)rows, (cuuint64_t)H, (cuuint64_t)outer};
      cuuint64_t strides[3] = {sl, sh, sb};
      cuuint32_t box[4] = {64, 128, 1, 1};
      cuuint32_t estr[4] = {1, 1, 1, 1};
      // the map depends only on the cache's address, dtype, extents and strides:
      // the last few are kept (a decode loop cycles over one cache per layer)
      const std::array<unsigned long long, 9> tkey = {(unsigned long long)reinterpret_cast<uintptr_t>(base),
                                                      (unsigned long long)a->dtype, dims[0], dims[1], dims[2], dims[3],
                                                      sl, sh, sb};
      static std::mutex tmu;
      static std::map<std::array<unsigned long long, 9>, CUtensorMap> tmaps;
      {
        std::lock_guard<std::mutex> lock(tmu);
        auto it = tmaps.find(tkey);
        if (it != tmaps.end()) {
          *out = it->second;
          return SAGA_OK;
        }
      }
      CUresult r = enc(out, a->dtype == SAGA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        *err = std::string("cuTensorMapEncodeTiled failed for the ") + what + " (" + std::to_string((int)r) + ")";
        return SAGA_ERR_INVALID;
      }
      std::lock_guard<std::mutex> lock(tmu);
      if (tmaps.size() >= 256) tmaps.clear();
      tmaps[tkey] = *out;
      return SAGA_OK;
    };
    int rc = encode(&p.tmap, a->k, a->Hk, a->k_sl, a->k_sh, a->k_sb, "key cache");
    if (rc != SAGA_OK) return rc;
    // dense steps on the tensor-core P.V stream the value tiles by TMA as well
    if (mode == MODE_DENSE && a->D == 128 && !paged) {
      rc = encode(&p.vmap, a->v, a->Hv, a->v_sl, a->v_sh, a->v_sb, "value cache");
      if (rc != SAGA_OK) return rc;
    }
  }

  const void* kfn = pick_kernel(a->dtype, a->D, mode, pl.tc, a->mask != nullptr, shards > 1, a->page_table != nullptr);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = pl.cooperative ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* kargs[] = {&p};
  cudaError_t e = cudaLaunchKernelExC(&cfg, kfn, kargs);
  if (e != cudaSuccess) {
    *err = std::string("kernel launch: ") + cudaGetErrorString(e);
    return SAGA_ERR_CUDA;
  }
  if (launched) {
    if (!launched->empty()) *launched += ",";
    *launched += mode_name(mode);
  }
  return SAGA_OK;
}

}  // namespace saga
