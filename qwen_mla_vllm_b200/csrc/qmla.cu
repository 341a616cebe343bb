// libqmla: C-ABI entry points (include/qmla.h) over the sm_100a kernels.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "qmla.h"
#include "qmla_aux.cuh"
#include "qmla_dcp.cuh"
#include "qmla_decode.cuh"

using namespace qmla;

namespace {

constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in limit per block on sm_100
constexpr int kMaxRing = 12;         // K / V ring slots at most (bounds the barrier area)

struct DevInfo {
  int sms = 0;
  int max_smem = 0;
  bool ok = false;
};

std::mutex g_mu;
std::map<int, DevInfo> g_dev;

DevInfo dev_info(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_dev.find(dev);
  if (it != g_dev.end()) return it->second;
  DevInfo d;
  if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) ==
          cudaSuccess)
    d.ok = true;
  g_dev[dev] = d;
  return d;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

using MapKey = std::tuple<const void*, int, int, int, int64_t, int64_t, int64_t, int, int>;
std::map<MapKey, CacheMaps> g_maps;

// The decode kernel's three maps over the paged cache (CacheMaps in qmla_decode.cuh):
//   chunk: 3-D (row element, token in page, page), box = one 128-byte column x `run`
//          tokens; the row extent is the QK width, so columns past it (rms tail,
//          padding) are zero-filled;
//   pair:  5-D (element of a 128-byte column, token in an 8-token group, column,
//          8-token group in the page, page), box = two columns x `run` tokens, which
//          lands as [8-token group][column][token][128 B]; the column extent counts the
//          full columns only;
//   vrows: the pair map's view with box = `vcols` columns x 16 tokens (V slots).
// Pages outside [0, num_pages) are zero-filled by all three.
int cache_tensor_map(const qmla_decode_params* p, int run, int vcols, CacheMaps* out) {
  const bool fp8 = p->kv_dtype == QMLA_DT_FP8E4M3;
  const int es = fp8 ? 1 : 2;
  MapKey key{p->kv_cache, p->kv_dtype, p->qk_dim, p->page_size, p->kv_num_pages,
             p->kv_stride_page, p->kv_stride_token, run, vcols};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return QMLA_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) return QMLA_E_CUDA;
  CUtensorMapDataType dt = fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int64_t tok_b = p->kv_stride_token * es, page_b = p->kv_stride_page * es;
  CacheMaps m;
  {
    cuuint64_t dims[3] = {(cuuint64_t)p->qk_dim, (cuuint64_t)p->page_size,
                          (cuuint64_t)p->kv_num_pages};
    cuuint64_t strides[2] = {(cuuint64_t)tok_b, (cuuint64_t)page_b};
    cuuint32_t box[3] = {(cuuint32_t)(128 / es), (cuuint32_t)run, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(&m.chunk, dt, 3, const_cast<void*>(p->kv_cache), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return QMLA_E_ALIGNMENT;
  }
  {
    const int full_chunks = p->qk_dim * es / 128;
    cuuint64_t dims[5] = {(cuuint64_t)(128 / es), 8, (cuuint64_t)full_chunks,
                          (cuuint64_t)(p->page_size / 8), (cuuint64_t)p->kv_num_pages};
    cuuint64_t strides[4] = {(cuuint64_t)tok_b, 128, (cuuint64_t)(8 * tok_b), (cuuint64_t)page_b};
    cuuint32_t box[5] = {(cuuint32_t)(128 / es), 8, 2, (cuuint32_t)(run / 8), 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(&m.pair, dt, 5, const_cast<void*>(p->kv_cache), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return QMLA_E_ALIGNMENT;
  }
  {
    const int full_chunks = p->qk_dim * es / 128;
    cuuint64_t dims[5] = {(cuuint64_t)(128 / es), 8, (cuuint64_t)full_chunks,
                          (cuuint64_t)(p->page_size / 8), (cuuint64_t)p->kv_num_pages};
    cuuint64_t strides[4] = {(cuuint64_t)tok_b, 128, (cuuint64_t)(8 * tok_b), (cuuint64_t)page_b};
    cuuint32_t box[5] = {(cuuint32_t)(128 / es), 8, (cuuint32_t)vcols, 2, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(&m.vrows, dt, 5, const_cast<void*>(p->kv_cache), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return QMLA_E_ALIGNMENT;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps[key] = m;
  *out = m;
  return QMLA_OK;
}

int gcd_int(int a, int b) {
  while (b) {
    int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Makes `dev` the current device for the lifetime of the guard and puts the caller's current
// device back on every return path, so an entry point never leaves a thread that drives several
// GPUs pointed at another one.
class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) return;
    if (prev_ == dev) {
      ok_ = true;
      return;
    }
    ok_ = cudaSetDevice(dev) == cudaSuccess;
    switched_ = ok_;
  }
  ~DeviceGuard() {
    if (switched_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int prev_ = -1;
  bool ok_ = false, switched_ = false;
};

struct Plan {
  int fold, R, work_rows;  // decode rows folded into one work row, its query rows, work rows
  int npv, nb, nqk;
  int use_tma, run;
  int n_qk_slots, n_sub_qk, n_full_chunks, cps;
  int v_tma;               // V slots by TMA boxes
  int v_blocks;            // V by TMA: output blocks per V slot
  uint32_t v_slot_bytes;   // bytes of a V slot
  int qk_bytes, row_bytes;
  int rms_bytes, rms_base_b, rms_units, rms_skip, pf_bytes;
  int G;
  int q_vec, qpe_vec;
  // workspace offsets
  int64_t ws_status, ws_bounds, ws_prefix, ws_done, ws_plse, ws_po, ws_qimg, ws_qscale, ws_total;
  int q_img_bytes;  // FP8: bytes of one work row's Q buffer image (0 for bf16)
  bool row_merge;  // rows cut at CTA boundaries are merged inside the decode kernel
  // smem
  uint32_t off_kring, nk, off_vring, nv, off_q, q_chunk, off_p, p_bytes, off_rms, off_misc;
  uint32_t smem_total;
};

constexpr int kMaxQueryRows = 48;  // query rows of a work row the kernel is built for

int make_plan_fold(const qmla_decode_params* p, Plan* pl, int fold) {
  if (!p || !p->q || !p->kv_cache || !p->block_table || !p->seq_lens || !p->o)
    return QMLA_E_INVALID;
  if (!p->q_pe && p->qk_dim > p->rank) return QMLA_E_INVALID;
  if (p->num_rows < 0 || p->num_heads <= 0 || p->num_heads > kMaxQueryRows) return QMLA_E_UNSUPPORTED;
  pl->fold = fold;
  pl->R = fold * p->num_heads;
  pl->work_rows = p->num_rows / fold;
  if (pl->R > kMaxQueryRows) return QMLA_E_UNSUPPORTED;
  if (p->rank <= 0 || p->rank % 128 != 0) return QMLA_E_UNSUPPORTED;
  const int nb = p->rank / 128;
  if (!(nb == 2 || nb == 3 || nb == 4 || nb == 6 || nb == 14)) return QMLA_E_UNSUPPORTED;
  if (p->qk_dim < p->rank || p->qk_dim > 2048) return QMLA_E_UNSUPPORTED;
  // rank 1792 (14 output blocks): O takes 14 x 32 TMEM columns, so at most 32 query rows
  if (nb == 14 && fold * p->num_heads > 32) return QMLA_E_UNSUPPORTED;
  if (p->page_size <= 0) return QMLA_E_INVALID;
  if (p->q_dtype != QMLA_DT_BF16 && p->q_dtype != QMLA_DT_F16) return QMLA_E_UNSUPPORTED;
  if (p->o_dtype < 0 || p->o_dtype > 2) return QMLA_E_UNSUPPORTED;
  if (p->lse && (p->lse_dtype < 0 || p->lse_dtype > 2)) return QMLA_E_UNSUPPORTED;
  const bool fp8 = p->kv_dtype == QMLA_DT_FP8E4M3;
  if (!fp8 && p->kv_dtype != QMLA_DT_BF16) return QMLA_E_UNSUPPORTED;  // f16 caches: not built
  if (p->rms_mode < 0 || p->rms_mode > 3) return QMLA_E_INVALID;
  if (!fp8 && p->rms_mode >= 2) return QMLA_E_INVALID;
  const int es = fp8 ? 1 : 2;
  if (reinterpret_cast<uintptr_t>(p->kv_cache) % 16 != 0) return QMLA_E_ALIGNMENT;
  if ((p->kv_stride_token * es) % 16 != 0 || (p->kv_stride_page * es) % 16 != 0)
    return QMLA_E_ALIGNMENT;
  if (p->kv_row_width < p->qk_dim || p->kv_stride_token < p->kv_row_width) return QMLA_E_INVALID;

  pl->nb = nb;
  pl->nqk = pl->R <= 16 ? 16 : pl->R <= 24 ? 24 : pl->R <= 32 ? 32 : 48;
  pl->npv = pl->nqk <= 16 ? 16 : pl->nqk <= 32 ? 32 : 48;
  // Pages holding whole runs of 16 tokens are loaded with TMA boxes (no shared
  // memory staging through L1); other page sizes with 16-byte cp.async gathers.
  pl->run = gcd_int(p->page_size, kTile);
  pl->use_tma = pl->run >= 16 ? 1 : 0;
  if (getenv("QMLA_NO_TMA")) pl->use_tma = 0;  // test hook: force the cp.async path
  pl->qk_bytes = p->qk_dim * es;
  pl->row_bytes = p->kv_row_width * es;
  // rms tail: bf16 values (bf16 cache, or FP8 cache in BF16 mode), else one byte per head
  pl->rms_bytes = p->rms_mode == QMLA_RMS_NONE ? 0
                  : (!fp8 || p->rms_mode == QMLA_RMS_BF16) ? 2 * p->num_heads
                                                           : p->num_heads;
  pl->rms_base_b = pl->rms_units = pl->rms_skip = 0;
  if (p->rms_mode != QMLA_RMS_NONE) {
    const int64_t off_b = (int64_t)p->rms_offset * es;
    if (p->rms_offset < p->qk_dim || off_b + pl->rms_bytes > pl->row_bytes) return QMLA_E_INVALID;
    pl->rms_base_b = (int)(off_b & ~int64_t(15));
    pl->rms_skip = (int)(off_b - pl->rms_base_b);
    pl->rms_units = (pl->rms_skip + pl->rms_bytes + 15) / 16;
    if (pl->rms_units > kRmsMaxUnits) return QMLA_E_UNSUPPORTED;
  }
  {
    // L2 prefetch span of a row: the QK columns and the rms tail, in 16-byte units
    int64_t end = pl->qk_bytes;
    if (pl->rms_units) end = std::max<int64_t>(end, pl->rms_base_b + 16 * pl->rms_units);
    end = std::min<int64_t>(align_up(end, 16), p->kv_stride_token * es);
    pl->pf_bytes = (int)end;
  }
  // K slots hold one or two 128-byte column chunks of each of the tile's 128 tokens.  Two
  // (paired layout, 4 KB TMA boxes) for rank 768 with up to 32 query rows: one lane-issued
  // TMA box costs ~70 ns whatever its size up to 4 KB, so 2 KB boxes held the K stream to
  // ~35 GB/s per SM against ~56 GB/s with 4 KB boxes (B200, boxes of random pages).
  pl->n_sub_qk = (pl->qk_bytes + 127) / 128;
  pl->n_full_chunks = pl->qk_bytes / 128;
  bool paired = pl->use_tma && nb == 6 && pl->nqk <= 32;
  if (getenv("QMLA_NO_PAIR")) paired = false;  // test hook: the one-column layout
  pl->cps = paired ? 2 : 1;
  pl->n_qk_slots = (pl->n_sub_qk + pl->cps - 1) / pl->cps;
  if (pl->n_sub_qk > kMaxQkChunks) return QMLA_E_UNSUPPORTED;
  // 16-byte vector loads of q rows (bf16 only; element strides in 2-byte units)
  auto vec_ok = [](const void* ptr, int64_t sr, int64_t sh) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (sr * 2) % 16 == 0 && (sh * 2) % 16 == 0;
  };
  pl->q_vec = p->q_dtype == QMLA_DT_BF16 && vec_ok(p->q, p->q_stride_row, p->q_stride_head);
  const void* qpe = p->q_pe ? p->q_pe : p->q;
  int64_t psr = p->q_pe ? p->qpe_stride_row : p->q_stride_row;
  int64_t psh = p->q_pe ? p->qpe_stride_head : p->q_stride_head;
  pl->qpe_vec = p->q_dtype == QMLA_DT_BF16 && vec_ok(qpe, psr, psh);

  DevInfo di = dev_info(p->device);
  if (!di.ok) return QMLA_E_CUDA;
  int G = p->num_ctas > 0 ? p->num_ctas : di.sms;
  G = std::min(G, kMaxCtas);
  pl->G = G;

  // shared memory map: K ring, V ring, Q, 2 P buffers, 2 rms staging buffers, misc
  const uint32_t kslot = 16384u * (uint32_t)pl->cps;  // 128 tokens x cps 128-byte columns
  const int q_rows = fp8 ? 2 * pl->nqk : pl->nqk;
  pl->q_chunk = (uint32_t)((q_rows + 7) / 8 * 1024);
  const uint32_t q_bytes = pl->q_chunk * pl->n_sub_qk;
  pl->p_bytes = (uint32_t)(pl->npv * 2 * kTile);  // P^T of a tile: bf16, or e4m3 hi + lo
  const uint32_t misc_bytes = 5120;
  const uint32_t rms_smem = (uint32_t)(2 * kTile * 16 * pl->rms_units);  // two staging buffers
  const uint32_t fixed = q_bytes + 2 * pl->p_bytes + misc_bytes + rms_smem + 1024 /*align slack*/;
  const int budget = std::min(di.max_smem, kMaxDynSmem) - (int)fixed;
  // V slots.  By TMA (bf16 caches with one-column K slots): one PV K step of tokens (16) x
  // v_blocks output blocks, 4 KB per block, filled by one box per 16 tokens; v_blocks = the
  // largest divisor of the block count with slots of at most 24 KB of which two fit beside
  // 64 KB of K slots (else beside one K slot).  By cp.async: 64 tokens x one block, filled by
  // three warps in turn (paired K slots) or two warps sharing each slot.  Measured on B200
  // against the cp.async fills: GLA rank 384 x 12 heads (config 3) 0.61 vs 0.74 ms per group;
  // config 1 (paired) 0.65 vs 0.63, e4m3 config 2 (48 query rows, 2 KB K boxes) 1.57 vs 1.35:
  // their K boxes queue behind the V boxes in the SM's TMA unit.
  // The V groups take the V slots in turn (slot n: group n % v_groups).  With at least as
  // many slots as groups, a group's wait for slot n's position to be free comes after its
  // own fill of slot n - v_groups, so the position is never two phases behind (a parity
  // wait would then pass early; with fewer slots than groups calls hung until the 2 s
  // wait limit).  Two slots at least, so a load overlaps the MMAs of the previous slot.
  pl->v_tma = pl->use_tma && !fp8 && !paired;
  // test hook: V copied by cp.async where the default is TMA boxes (the kernels that take
  // boxes are built for bf16 with one-column K slots only)
  if (const char* e = getenv("QMLA_V_TMA")) pl->v_tma = pl->v_tma && atoi(e) != 0;
  const int nv_min = pl->v_tma ? 2 : std::max(2, paired ? 3 : 1);
  pl->v_blocks = nb;
  uint32_t vslot = fp8 ? 8192u : 16384u;
  int v_per_tile = 2 * nb;  // V slots per tile
  if (pl->v_tma) {
    int vb = 0;
    for (int kr : {std::max<int>((int)kslot, 65536), (int)kslot})
      for (int d = nb; d >= 1 && !vb; --d)
        if (nb % d == 0 && 4096 * d <= 24576 && budget >= kr + nv_min * 4096 * d) vb = d;
    if (const char* e = getenv("QMLA_VB")) {  // test hook: blocks per V slot (a legal divisor)
      const int d = atoi(e);
      if (d >= 1 && d <= nb && nb % d == 0 && budget >= (int)kslot + nv_min * 4096 * d) vb = d;
    }
    if (!vb) return QMLA_E_UNSUPPORTED;
    pl->v_blocks = vb;
    vslot = 4096u * (uint32_t)vb;
    v_per_tile = (kTile / (fp8 ? 32 : 16)) * (nb / vb);
  }
  pl->v_slot_bytes = vslot;
  if (budget < (int)(kslot + nv_min * vslot)) return QMLA_E_UNSUPPORTED;
  // K ring: the HBM stream (bandwidth x latency), ~55% of the rings; V ring: L2 re-reads for PV
  const int nk_max = (budget - nv_min * (int)vslot) / (int)kslot;
  int nk = std::min(((budget * 11 / 20) + (int)kslot - 1) / (int)kslot, 3 * pl->n_qk_slots);
  if (paired) nk = 2;  // 64 KB of K, the rest for V
  nk = std::max(1, std::min({nk, nk_max, kMaxRing}));
  // test hooks: QMLA_NK / QMLA_NV override the ring sizes (clamped to legal values)
  if (const char* e = getenv("QMLA_NK")) nk = std::max(1, std::min({atoi(e), nk_max, kMaxRing}));
  int nv = std::min({(budget - nk * (int)kslot) / (int)vslot, 2 * v_per_tile, kMaxRing});
  if (const char* e = getenv("QMLA_NV")) nv = std::min(atoi(e), nv);
  nv = std::max(nv, nv_min);
  if (nk * (int)kslot + nv * (int)vslot > budget) return QMLA_E_UNSUPPORTED;
  pl->nk = (uint32_t)nk;
  pl->nv = (uint32_t)nv;
  // barriers, abort flag + TMEM slot, red[256] + hv[256] floats, tokptr[2][kTile]
  const uint32_t n_bars = 2 * (pl->nk + pl->nv) + 14 + kKdoneDepth + 4;
  if ((n_bars * 8 + 15) / 16 * 16 + 16 + 1024 + 1024 + 16 * kTile > misc_bytes)
    return QMLA_E_UNSUPPORTED;
  uint32_t off = 0;
  pl->off_kring = off;
  off += pl->nk * kslot;
  pl->off_vring = off;
  off += pl->nv * vslot;
  pl->off_q = off;
  off += q_bytes;
  pl->off_p = off;
  off += 2 * pl->p_bytes;
  pl->off_rms = off;
  off += rms_smem;
  pl->off_misc = (uint32_t)align_up(off, 16);
  off = pl->off_misc + misc_bytes;
  pl->smem_total = off + 1024;

  // workspace map
  int64_t w = 0;
  pl->ws_status = w;
  w += 256;
  pl->ws_bounds = w;
  w = align_up(w + 4 * ((int64_t)kMaxCtas + 1), 256);
  pl->ws_prefix = w;
  w = align_up(w + 4 * ((int64_t)pl->work_rows + 1), 256);
  // Rows cut at CTA boundaries are merged by the merge kernel, spread over (row, query row)
  // blocks.  Merging them inside the decode kernel (the CTA that finishes a row's last piece
  // merges it; test hook QMLA_ROW_MERGE, for calls with at least a quarter as many rows as CTAs)
  // saves that launch but puts the merge on the slowest CTA's path: config 1 measured 0.647 ms
  // against 0.621 with the merge kernel.
  pl->row_merge = (int64_t)pl->work_rows * 4 >= G && getenv("QMLA_ROW_MERGE") != nullptr;
  pl->ws_done = w;
  w = align_up(w + 4 * (int64_t)pl->work_rows, 256);
  pl->ws_plse = w;
  w = align_up(w + 4 * (int64_t)2 * G * pl->R, 256);
  pl->ws_po = w;
  w = align_up(w + 4 * (int64_t)2 * G * pl->R * p->rank, 256);
  // FP8: every work row's Q buffer image and q scales, written by q_fp8_prep_kernel
  pl->q_img_bytes = fp8 ? (int)q_bytes : 0;
  pl->ws_qimg = w;
  w = align_up(w + (int64_t)pl->q_img_bytes * pl->work_rows, 256);
  pl->ws_qscale = w;
  w = align_up(w + (fp8 ? 4 * (int64_t)pl->nqk * pl->work_rows : 0), 256);
  pl->ws_total = w;
  return QMLA_OK;
}

// MTP verify (qrows > 1, rows flattened per request): fold the largest divisor F of qrows with
// F * heads <= 48 drafts into one work row, so the request's cache is read qrows / F times
// instead of qrows times.  Falls back to one decode row per work row where the folded shape does
// not fit (shared memory), or when allow_fold is false (test hook QMLA_NO_FOLD: never fold).
// Measured on B200 with 4 drafts x 8192 tokens: bf16 rank 768 x 24 heads 0.74 ms folded vs
// 1.04 unfolded; FP8 rank 384 x 12 heads 1.04 vs 1.52; bf16 rank 384 x 12 heads 0.89 vs 1.47;
// FP8 rank 768 x 24 heads 1.38 vs 1.48.
int make_plan(const qmla_decode_params* p, Plan* pl, bool allow_fold = true) {
  int fold = 1;
  if (p && allow_fold && p->qrows > 1 && p->num_rows % p->qrows == 0 && !getenv("QMLA_NO_FOLD")) {
    for (int f = p->qrows; f >= 2; --f)
      if (p->qrows % f == 0 && f * p->num_heads <= kMaxQueryRows) {
        fold = f;
        break;
      }
  }
  int rc = make_plan_fold(p, pl, fold);
  if (rc == QMLA_E_UNSUPPORTED && fold > 1) rc = make_plan_fold(p, pl, 1);
  return rc;
}

template <bool FP8, int NB, int NQK, bool PAIR>
int launch_decode_t(const CacheMaps& maps, const DecodeArgs& a, uint32_t smem,
                    cudaStream_t st) {
  auto k = mla_decode_kernel<FP8, NB, NQK, PAIR>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  static bool regs_ok = true;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if constexpr (NQK >= 32) {
      // the warpgroups' setmaxnreg budgets add up to exactly the pool of a CTA launched with
      // kRegsAtLaunch registers per thread; with fewer, a setmaxnreg.inc would wait forever, so
      // such a build is never launched
      cudaFuncAttributes fa;
      // (registers are allocated to a warp in units of 8 per thread)
      regs_ok = attr_err == cudaSuccess && cudaFuncGetAttributes(&fa, k) == cudaSuccess &&
                (fa.numRegs + 7) / 8 * 8 * kNumThreads >= (int)(kRegsSoftmax + kRegsProducer) * 256;
    }
  });
  if (attr_err != cudaSuccess) return QMLA_E_CUDA;
  if (!regs_ok) return QMLA_E_UNSUPPORTED;
  k<<<a.G, kNumThreads, smem, st>>>(maps, a);
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

template <bool FP8, int NB, bool PAIR>
int launch_decode_nb(int nqk, const CacheMaps& maps, const DecodeArgs& a, uint32_t smem,
                     cudaStream_t st) {
  switch (nqk) {
    case 16:
      return launch_decode_t<FP8, NB, 16, PAIR>(maps, a, smem, st);
    case 24:
      return launch_decode_t<FP8, NB, 24, PAIR>(maps, a, smem, st);
    case 32:
      return launch_decode_t<FP8, NB, 32, PAIR>(maps, a, smem, st);
    case 48:
      if constexpr (!PAIR && NB * 48 <= 448) return launch_decode_t<FP8, NB, 48, false>(maps, a, smem, st);
      break;
  }
  return QMLA_E_UNSUPPORTED;
}

template <bool FP8>
int launch_decode_fp(int nb, int nqk, const CacheMaps& maps, const DecodeArgs& a,
                     uint32_t smem, cudaStream_t st) {
  switch (nb) {
    case 2:
      return launch_decode_nb<FP8, 2, false>(nqk, maps, a, smem, st);
    case 3:
      return launch_decode_nb<FP8, 3, false>(nqk, maps, a, smem, st);
    case 4:
      return launch_decode_nb<FP8, 4, false>(nqk, maps, a, smem, st);
    case 6:
      return launch_decode_nb<FP8, 6, false>(nqk, maps, a, smem, st);
    case 14:
      return launch_decode_nb<FP8, 14, false>(nqk, maps, a, smem, st);
  }
  return QMLA_E_UNSUPPORTED;
}

// paired K slots: instantiated for rank 768 (the planner's choice)
int launch_decode(bool fp8, bool paired, int nb, int nqk, const CacheMaps& maps,
                  const DecodeArgs& a, uint32_t smem, cudaStream_t st) {
  if (paired) {
    if (nb != 6) return QMLA_E_UNSUPPORTED;
    return fp8 ? launch_decode_nb<true, 6, true>(nqk, maps, a, smem, st)
               : launch_decode_nb<false, 6, true>(nqk, maps, a, smem, st);
  }
  return fp8 ? launch_decode_fp<true>(nb, nqk, maps, a, smem, st)
             : launch_decode_fp<false>(nb, nqk, maps, a, smem, st);
}

#ifdef QMLA_TRACE
unsigned long long* g_trace = nullptr;
#endif

// Scratch for qmla_mla_decode_static: a fixed device array instead of a caller workspace.
// A call fits when qmla_decode_workspace_bytes() <= 32 MiB.  The per-CTA fp32 partials take the
// most: at the largest shape (160 CTAs x 32 heads x rank 768, 31.5 MB of partials) about 513,000
// rows still fit; at one CTA per B200 SM with 24 heads and rank 768, about 2.9 million.  Every GPU
// that loads the library holds one copy until the process exits, shared by every call on it.
constexpr int64_t kStaticScratchBytes = int64_t(32) << 20;
__device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];
std::map<int, void*> g_static_addr;  // device -> address of g_static_scratch (looked up once)

void* static_scratch(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_static_addr.find(dev);
  if (it != g_static_addr.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess) return nullptr;
  g_static_addr[dev] = p;
  return p;
}

}  // namespace

extern "C" {

#ifdef QMLA_TRACE
// Diagnostic builds only: stage timestamps of CTA 0 go to this device buffer.
void qmla_set_trace(void* dev_ptr) { g_trace = reinterpret_cast<unsigned long long*>(dev_ptr); }
#endif

int qmla_abi_version(void) { return 103; }

const char* qmla_error_string(int code) {
  switch (code) {
    case QMLA_OK:
      return "ok";
    case QMLA_E_INVALID:
      return "invalid argument";
    case QMLA_E_UNSUPPORTED:
      return "unsupported shape or dtype";
    case QMLA_E_ALIGNMENT:
      return "pointer or stride not 16-byte aligned";
    case QMLA_E_WORKSPACE:
      return "workspace too small";
    case QMLA_E_CUDA:
      return "CUDA call failed";
    case QMLA_E_DEVICE_TIMEOUT:
      return "device wait timed out";
    default:
      return "unknown error";
  }
}

int qmla_decode_workspace_bytes(const qmla_decode_params* p, int64_t* bytes) {
  if (!bytes) return QMLA_E_INVALID;
  Plan pl;
  int rc = make_plan(p, &pl);
  if (rc != QMLA_OK) return rc;
  *bytes = pl.ws_total;
  return QMLA_OK;
}

}  // extern "C"

namespace {
// qmla_mla_decode with the folding choice exposed (the static-scratch entry point turns folding
// off when the folded partials would not fit its array).
int decode_impl(const qmla_decode_params* p, void* stream, bool allow_fold) {
  Plan pl;
  int rc = make_plan(p, &pl, allow_fold);
  if (rc != QMLA_OK) return rc;
  if (!p->workspace || p->workspace_bytes < pl.ws_total) return QMLA_E_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(p->workspace) % 256 != 0) return QMLA_E_ALIGNMENT;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DeviceGuard dg(p->device);
  if (!dg.ok()) return QMLA_E_CUDA;

  uint8_t* ws = reinterpret_cast<uint8_t*>(p->workspace);
  DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.q = reinterpret_cast<const uint8_t*>(p->q);
  a.q_pe = reinterpret_cast<const uint8_t*>(p->q_pe ? p->q_pe : p->q);
  a.q_sr = p->q_stride_row;
  a.q_sh = p->q_stride_head;
  a.qpe_sr = p->q_pe ? p->qpe_stride_row : p->q_stride_row;
  a.qpe_sh = p->q_pe ? p->qpe_stride_head : p->q_stride_head;
  a.q_dtype = p->q_dtype;
  a.q_vec = pl.q_vec;
  a.qpe_vec = pl.qpe_vec;
  a.block_table = p->block_table;
  a.bt_stride = p->block_table_stride;
  a.seq_lens = p->seq_lens;
  a.page_size = p->page_size;
  a.use_tma = pl.use_tma;
  a.run_rows = pl.run;
  a.cache = reinterpret_cast<const uint8_t*>(p->kv_cache);
  {
    const int es = p->kv_dtype == QMLA_DT_FP8E4M3 ? 1 : 2;
    a.page_stride_b = p->kv_stride_page * es;
    a.token_stride_b = p->kv_stride_token * es;
    a.num_pages = p->kv_num_pages;
  }
  a.num_rows = pl.work_rows;
  a.fold = pl.fold;
  a.R = pl.R;
  a.H = p->num_heads;
  a.rank = p->rank;
  a.qk_dim = p->qk_dim;
  a.rms_mode = p->rms_mode;
  a.qk_bytes = pl.qk_bytes;
  a.row_bytes = pl.row_bytes;
  a.n_qk_slots = pl.n_qk_slots;
  a.n_sub_qk = pl.n_sub_qk;
  a.n_full_chunks = pl.n_full_chunks;
  // a row segment's fixed overhead, in tiles, for the work partition (test hook QMLA_SEG_COST)
  a.seg_cost = 2;  // swept 0-4: 2 best on a DCP rank's shard (+17% over 0), config 1 and GLA flat
  if (const char* e = getenv("QMLA_SEG_COST")) a.seg_cost = std::max(0, std::min(atoi(e), 64));
  a.early_q = kEarlyQTiles;  // test hook QMLA_EARLY_Q: the longest segment that stages Q early
  if (const char* e = getenv("QMLA_EARLY_Q")) a.early_q = std::max(0, atoi(e));

  a.rms_base_b = pl.rms_base_b;
  a.rms_units = pl.rms_units;
  a.rms_skip = pl.rms_skip;
  a.pf_bytes = pl.pf_bytes;
  a.sm_scale = p->sm_scale;
  a.logit_cap = p->logit_cap;
  a.k_scale = p->k_scale;
  a.o = reinterpret_cast<uint8_t*>(p->o);
  a.o_sr = p->o_stride_row;
  a.o_sh = p->o_stride_head;
  a.o_dtype = p->o_dtype;
  a.lse = reinterpret_cast<uint8_t*>(p->lse);
  a.lse_sr = p->lse_stride_row;
  a.lse_dtype = p->lse_dtype;
  a.status = reinterpret_cast<int*>(ws + pl.ws_status);
  // a host plan (qmla_plan) is per decode row: used only when rows are not folded
  const int32_t* host_prefix = pl.fold == 1 ? p->plan_tile_prefix : nullptr;
  a.tile_prefix = host_prefix ? host_prefix : reinterpret_cast<const int32_t*>(ws + pl.ws_prefix);
  a.part_lse = reinterpret_cast<float*>(ws + pl.ws_plse);
  a.range_bounds = reinterpret_cast<const int32_t*>(ws + pl.ws_bounds);
  a.part_o = reinterpret_cast<float*>(ws + pl.ws_po);
  a.q_img = ws + pl.ws_qimg;
  a.q_scale = reinterpret_cast<const float*>(ws + pl.ws_qscale);
  a.q_img_bytes = pl.q_img_bytes;
  a.row_done = pl.row_merge ? reinterpret_cast<int*>(ws + pl.ws_done) : nullptr;
  a.G = pl.G;
  a.off_kring = pl.off_kring;
  a.nk = pl.nk;
  a.off_vring = pl.off_vring;
  a.nv = pl.nv;
  a.off_q = pl.off_q;
  a.q_chunk_bytes = pl.q_chunk;
  a.v_tma = pl.v_tma;
  a.v_blocks = pl.v_blocks;
  a.v_slot_bytes = pl.v_slot_bytes;
  a.off_p = pl.off_p;
  a.p_bytes = pl.p_bytes;
  a.off_rms = pl.off_rms;
  a.off_misc = pl.off_misc;
#ifdef QMLA_TRACE
  a.trace = g_trace;
  a.trace_cta = getenv("QMLA_TRACE_CTA") ? (unsigned)atoi(getenv("QMLA_TRACE_CTA")) : 0u;
  a.trace_tid = getenv("QMLA_TRACE_TID") ? atoi(getenv("QMLA_TRACE_TID")) : 0;
#else
  a.trace = nullptr;
#endif

  if (p->num_rows == 0) return QMLA_OK;
  CacheMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (pl.use_tma) {
    rc = cache_tensor_map(p, pl.run, pl.v_blocks * (p->kv_dtype == QMLA_DT_FP8E4M3 ? 1 : 2), &maps);
    if (rc != QMLA_OK) return rc;
  }
  int32_t* bounds = reinterpret_cast<int32_t*>(ws + pl.ws_bounds);
  if (!host_prefix) {
    plan_kernel<<<1, 1024, 0, st>>>(p->seq_lens, pl.work_rows, pl.fold,
                                    reinterpret_cast<int32_t*>(ws + pl.ws_prefix), a.status,
                                    a.G, a.seg_cost, bounds, a.row_done);
  } else {
    bounds_kernel<<<1, 256, 0, st>>>(host_prefix, p->num_rows, a.status, a.G, a.seg_cost, bounds,
                                     a.row_done);
  }
  if (cudaGetLastError() != cudaSuccess) return QMLA_E_CUDA;
  if (pl.q_img_bytes > 0 && pl.work_rows > 0) {
    q_fp8_prep_kernel<<<dim3(pl.work_rows, pl.nqk), 128, 0, st>>>(a, pl.nqk, ws + pl.ws_qimg,
                                                                   reinterpret_cast<float*>(ws + pl.ws_qscale));
    if (cudaGetLastError() != cudaSuccess) return QMLA_E_CUDA;
  }
  rc = launch_decode(p->kv_dtype == QMLA_DT_FP8E4M3, pl.cps == 2, pl.nb, pl.nqk, maps, a,
                     pl.smem_total, st);
  if (rc != QMLA_OK) return rc;
  if (!pl.row_merge) {
    // few (row, query row) blocks: split the output dims over blocks too, so the merge has
    // enough blocks in flight (config 4: 192 blocks -> 1152)
    const int zsplit = (int64_t)pl.work_rows * pl.R < 1024 ? p->rank / 128 : 1;
    split_merge_kernel<<<dim3(pl.work_rows, pl.R, zsplit), 128, 0, st>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}
}  // namespace

extern "C" {

int qmla_mla_decode(const qmla_decode_params* p, void* stream) {
  return decode_impl(p, stream, true);
}

int qmla_mla_decode_static(const qmla_decode_params* p, void* stream) {
  if (!p) return QMLA_E_INVALID;
  Plan pl;
  int rc = make_plan(p, &pl, true);
  if (rc != QMLA_OK) return rc;
  // MTP folding widens the per-CTA partials (fold x heads query rows); where that would not fit
  // the array, decode the rows unfolded (same results, more cache reads)
  bool allow_fold = true;
  if (pl.ws_total > kStaticScratchBytes && pl.fold > 1) {
    allow_fold = false;
    rc = make_plan(p, &pl, false);
    if (rc != QMLA_OK) return rc;
  }
  if (pl.ws_total > kStaticScratchBytes) return QMLA_E_WORKSPACE;
  DeviceGuard dg(p->device);
  if (!dg.ok()) return QMLA_E_CUDA;
  void* scratch = static_scratch(p->device);
  if (!scratch) return QMLA_E_CUDA;
  // Same launch sequence as qmla_mla_decode.  The status word is the only scratch that must
  // start at zero: plan_kernel clears it, or bounds_kernel when a precomputed plan is given.
  // Everything else a call reads from the array it has written earlier in the same call.
  qmla_decode_params q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kStaticScratchBytes;
  return decode_impl(&q, stream, allow_fold);
}

int qmla_static_read_status(int32_t device, void* stream, int32_t* status) {
  if (!status) return QMLA_E_INVALID;
  DeviceGuard dg(device);
  if (!dg.ok()) return QMLA_E_CUDA;
  void* scratch = static_scratch(device);
  if (!scratch) return QMLA_E_CUDA;
  return qmla_read_status(scratch, stream, status);
}

int qmla_read_status(const void* workspace, void* stream, int32_t* status) {
  if (!workspace || !status) return QMLA_E_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return QMLA_E_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return QMLA_E_CUDA;
  return QMLA_OK;
}

int qmla_plan(const int32_t* seq_lens_host, int32_t num_rows, int32_t page_size,
              int32_t* tile_prefix, int32_t* kv_indptr, int32_t* kv_len, int64_t* total_tiles,
              int64_t* total_pages) {
  if (!seq_lens_host || !tile_prefix || num_rows < 0 || page_size <= 0) return QMLA_E_INVALID;
  int64_t t = 0, pg = 0;
  tile_prefix[0] = 0;
  if (kv_indptr) kv_indptr[0] = 0;
  for (int i = 0; i < num_rows; ++i) {
    int L = seq_lens_host[i] > 0 ? seq_lens_host[i] : 0;
    t += (L + kTile - 1) / kTile;
    pg += (L + page_size - 1) / page_size;
    if (t > INT32_MAX || pg > INT32_MAX) return QMLA_E_UNSUPPORTED;
    tile_prefix[i + 1] = (int32_t)t;
    if (kv_indptr) kv_indptr[i + 1] = (int32_t)pg;
    if (kv_len) kv_len[i] = L;
  }
  if (total_tiles) *total_tiles = t;
  if (total_pages) *total_pages = pg;
  return QMLA_OK;
}

int qmla_dcp_correct(void* out, int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                     const float* lses, int64_t lses_stride_n, int64_t lses_stride_b,
                     float* lse_out, int32_t n_ranks, int32_t cp_rank, int32_t B, int32_t H,
                     int32_t D, int32_t is_base_e, void* stream) {
  if (!out || !lses || n_ranks <= 0 || cp_rank < 0 || cp_rank >= n_ranks || B < 0 || H <= 0 ||
      D <= 0 || out_dtype < 0 || out_dtype > 2)
    return QMLA_E_INVALID;
  if (B == 0) return QMLA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dcp_correct_kernel<<<dim3(B, H), 128, 0, st>>>(reinterpret_cast<uint8_t*>(out), out_dtype,
                                                 out_stride_b, out_stride_h, lses, lses_stride_n,
                                                 lses_stride_b, lse_out, n_ranks, cp_rank, H, D,
                                                 is_base_e);
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_dcp_merge(const void* parts, int32_t parts_dtype, const float* part_lse, void* o,
                   int32_t o_dtype, float* lse, int32_t n_parts, int32_t B, int32_t H, int32_t D,
                   void* stream) {
  if (!parts || !part_lse || !o || n_parts <= 0 || n_parts > 64 || B < 0 || H <= 0 || D <= 0 ||
      parts_dtype < 0 || parts_dtype > 2 || o_dtype < 0 || o_dtype > 2)
    return QMLA_E_INVALID;
  if (B == 0) return QMLA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dcp_merge_kernel<<<dim3(B, H), 128, 0, st>>>(reinterpret_cast<const uint8_t*>(parts),
                                               parts_dtype, part_lse,
                                               reinterpret_cast<uint8_t*>(o), o_dtype, lse,
                                               n_parts, B, H, D);
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_dcp_buffer_layout(int32_t B, int32_t H, int32_t D, int64_t* total_bytes,
                           int64_t* o_offset, int64_t* o_slot_bytes, int64_t* lse_offset,
                           int64_t* lse_slot_bytes) {
  if (B < 0 || H <= 0 || D <= 0 || !total_bytes) return QMLA_E_INVALID;
  const ExchangeLayout L = ExchangeLayout::make(B, H, D);
  *total_bytes = L.total;
  if (o_offset) *o_offset = kDcpHeader;
  if (o_slot_bytes) *o_slot_bytes = L.o_slot;
  if (lse_offset) *lse_offset = L.lse_off;
  if (lse_slot_bytes) *lse_slot_bytes = L.lse_slot;
  return QMLA_OK;
}

int qmla_dcp_buffer_alloc(int32_t device, int64_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes < kDcpHeader) return QMLA_E_INVALID;
  *ptr = nullptr;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return QMLA_E_CUDA;
  if (cur != device && cudaSetDevice(device) != cudaSuccess) return QMLA_E_CUDA;
  void* p = nullptr;
  int rc = QMLA_OK;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) {
    rc = QMLA_E_CUDA;
  } else if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess ||
             cudaDeviceSynchronize() != cudaSuccess ||
             cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p) !=
                 cudaSuccess) {
    cudaFree(p);
    p = nullptr;
    rc = QMLA_E_CUDA;
  }
  *ptr = p;
  if (cur != device) cudaSetDevice(cur);
  return rc;
}

int qmla_dcp_buffer_open(int32_t device, const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return QMLA_E_INVALID;
  *ptr = nullptr;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return QMLA_E_CUDA;
  if (cur != device && cudaSetDevice(device) != cudaSuccess) return QMLA_E_CUDA;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (cur != device) cudaSetDevice(cur);
  return e == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_dcp_buffer_close(void* ptr) {
  if (!ptr) return QMLA_E_INVALID;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_dcp_buffer_free(void* ptr) {
  if (!ptr) return QMLA_E_INVALID;
  return cudaFree(ptr) == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_dcp_p2p_merge(const qmla_dcp_p2p_params* p, void* stream) {
  if (!p || p->world < 1 || p->world > kDcpMaxWorld || p->rank < 0 || p->rank >= p->world ||
      p->num_rows < 0 || p->num_heads <= 0 || p->head_dim <= 0 || p->head_dim % 4 != 0 ||
      !p->out || p->out_dtype < 0 || p->out_dtype > 2 ||
      (p->mode != QMLA_DCP_ALL_HEADS && p->mode != QMLA_DCP_HEAD_SCATTER))
    return QMLA_E_INVALID;
  if (p->mode == QMLA_DCP_HEAD_SCATTER && p->num_heads % p->world != 0) return QMLA_E_INVALID;
  for (int n = 0; n < p->world; ++n)
    if (!p->bufs[n] || reinterpret_cast<uintptr_t>(p->bufs[n]) % 256 != 0) return QMLA_E_INVALID;
  if (p->num_rows == 0) return QMLA_OK;
  DevInfo di = dev_info(p->device);
  if (!di.ok) return QMLA_E_CUDA;
  P2PArgs a;
  memset(&a, 0, sizeof(a));
  for (int n = 0; n < p->world; ++n) a.bufs[n] = reinterpret_cast<uint8_t*>(p->bufs[n]);
  a.world = p->world;
  a.rank = p->rank;
  a.B = p->num_rows;
  a.H = p->num_heads;
  a.D = p->head_dim;
  a.mode = p->mode;
  a.epoch = p->epoch;
  a.out = reinterpret_cast<uint8_t*>(p->out);
  a.out_sr = p->out_stride_row;
  a.out_sh = p->out_stride_head;
  a.out_dtype = p->out_dtype;
  a.lse_out = p->lse_out;
  a.timeout_ns = p->timeout_ns > 0 ? p->timeout_ns : 2000000000ll;
  const int hs = p->mode == QMLA_DCP_HEAD_SCATTER ? p->num_heads / p->world : p->num_heads;
  const int64_t items = (int64_t)p->num_rows * hs;
  const int grid = (int)std::min<int64_t>(items, 4 * (int64_t)di.sms);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dcp_p2p_merge_kernel<<<grid, 128, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_dcp_read_status(const void* buffer, void* stream, int32_t* status) {
  if (!buffer || !status) return QMLA_E_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const uint8_t* src = reinterpret_cast<const uint8_t*>(buffer) + 4 * kDcpMaxWorld;
  if (cudaMemcpyAsync(status, src, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return QMLA_E_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return QMLA_E_CUDA;
  return QMLA_OK;
}

int qmla_fp8_cache_write(const void* latent, int64_t latent_stride, const void* k_pe,
                         int64_t k_pe_stride, const int64_t* slot_mapping, int32_t n_tokens,
                         int32_t rank, int32_t rope, int32_t heads, int32_t rms_mode,
                         const float* k_scale, void* cache, int64_t cache_row_stride,
                         void* stream) {
  if (!latent || !k_pe || !slot_mapping || !cache || n_tokens < 0 || rank <= 0 || rope < 0 ||
      heads <= 0 || (rms_mode != QMLA_RMS_LOG8 && rms_mode != QMLA_RMS_BF16))
    return QMLA_E_INVALID;
  int rb = rms_mode == QMLA_RMS_LOG8 ? heads : 2 * heads;
  if (cache_row_stride < rank + rope + rb) return QMLA_E_INVALID;
  if (n_tokens == 0) return QMLA_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  fp8_cache_write_kernel<<<n_tokens, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(latent), latent_stride,
      reinterpret_cast<const __nv_bfloat16*>(k_pe), k_pe_stride, slot_mapping, rank, rope, heads,
      rms_mode, k_scale, reinterpret_cast<uint8_t*>(cache), cache_row_stride);
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

int qmla_gather_cache(const qmla_gather_params* p, void* stream) {
  if (!p || p->num_tokens < 0 || p->num_seqs < 0) return QMLA_E_INVALID;
  if (p->num_tokens == 0) return QMLA_OK;
  if (!p->src_cache || !p->dst || !p->block_table || !p->cu_seq_lens || !p->token_to_seq ||
      p->page_size <= 0 || p->num_pages <= 0 || p->block_table_cols <= 0 ||
      p->src_stride_page < 0 || p->src_stride_token < 0 || p->dst_stride_row < 0)
    return QMLA_E_INVALID;
  if (p->dst_dtype != QMLA_DT_BF16 && p->dst_dtype != QMLA_DT_F16 && p->dst_dtype != QMLA_DT_F32)
    return QMLA_E_UNSUPPORTED;
  const bool fp8 = p->src_dtype == QMLA_DT_FP8E4M3;
  if (!fp8 && p->src_dtype != QMLA_DT_BF16 && p->src_dtype != QMLA_DT_F16) return QMLA_E_UNSUPPORTED;
  GatherArgs a;
  memset(&a, 0, sizeof(a));
  const int se = fp8 ? 1 : 2, de = p->dst_dtype == QMLA_DT_F32 ? 4 : 2;
  int64_t src_row = 0, dst_cols = 0;
  if (fp8) {
    if (p->rms_offset <= 0 || p->rms_heads < 0 || !p->scale) return QMLA_E_INVALID;
    if (p->rms_mode == QMLA_RMS_NATIVE) {
      a.n_e4m3 = p->rms_offset + p->rms_heads;
      src_row = a.n_e4m3;
    } else if (p->rms_mode == QMLA_RMS_LOG8 || p->rms_mode == QMLA_RMS_BF16) {
      a.n_e4m3 = p->rms_offset;
      a.rms_heads = p->rms_heads;
      a.rms_off = p->rms_offset;
      a.rms_mode = p->rms_mode;
      src_row = p->rms_offset + (p->rms_mode == QMLA_RMS_BF16 ? 2 : 1) * (int64_t)p->rms_heads;
    } else {
      return QMLA_E_INVALID;
    }
    dst_cols = p->rms_offset + p->rms_heads;
  } else {
    if (p->row_elems <= 0) return QMLA_E_INVALID;
    a.n_copy = p->row_elems;
    src_row = dst_cols = p->row_elems;
  }
  if (p->src_stride_token < src_row || p->dst_stride_row < dst_cols) return QMLA_E_INVALID;
  a.src = reinterpret_cast<const uint8_t*>(p->src_cache);
  a.src_sp = p->src_stride_page * se;
  a.src_st = p->src_stride_token * se;
  a.page_size = p->page_size;
  a.num_pages = p->num_pages;
  a.bt = p->block_table;
  a.bt_stride = p->block_table_stride;
  a.bt_cols = p->block_table_cols;
  a.cu = p->cu_seq_lens;
  a.t2s = p->token_to_seq;
  a.starts = p->seq_starts;
  a.num_seqs = p->num_seqs;
  a.num_tokens = p->num_tokens;
  a.dst = reinterpret_cast<uint8_t*>(p->dst);
  a.dst_sr = p->dst_stride_row * de;
  a.dst_dt = p->dst_dtype;
  a.src_dt = p->src_dtype;
  a.scale = fp8 ? p->scale : nullptr;
  a.status = p->status;
  // 16-byte vector path when every source and destination row starts 16-byte aligned
  const bool vec = reinterpret_cast<uintptr_t>(a.src) % 16 == 0 && a.src_sp % 16 == 0 &&
                   a.src_st % 16 == 0 && reinterpret_cast<uintptr_t>(a.dst) % 16 == 0 &&
                   a.dst_sr % 16 == 0;
  DevInfo di = dev_info(p->device);
  if (!di.ok) return QMLA_E_CUDA;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Aligned rows: the staged kernel (whole rows by the bulk-copy engine through a shared-memory
  // ring), as many blocks as are resident at once.
  BulkShape bs;
  bs.copy_bytes = (int)(src_row / 16 * 16);
  bs.slot = bs.copy_bytes;
  // A 6-deep ring of 16 rows (8 when 16 would take more than ~100 KB of shared memory).  Swept
  // on the FP8 log8 bench shape: 16 x 6 gave 4.96 TB/s, 8 x 6 4.91, 8 x 4 4.73-4.82,
  // 32 x 3 4.58; a deeper ring counted for more than more blocks per SM.
  bs.stages = 6;
  bs.rows = 16;
  if (bulk_smem_bytes(bs) > 100 * 1024) bs.rows = 8;
  if (const char* e = getenv("QMLA_GATHER_ROWS"))  // test hook: rows per stage (8, 16, 24, 32)
    bs.rows = std::min(32, std::max(8, atoi(e) / 8 * 8));
  if (const char* e = getenv("QMLA_GATHER_STAGES"))  // test hook: ring depth (2..8)
    bs.stages = std::min(8, std::max(2, atoi(e)));
  if (vec && bs.copy_bytes >= 16 && bulk_smem_bytes(bs) <= 200 * 1024 &&
      getenv("QMLA_GATHER_REGS") == nullptr) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
      attr_err = cudaFuncSetAttribute(gather_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kMaxDynSmem);
    });
    if (attr_err != cudaSuccess) return QMLA_E_CUDA;
    const int smem = bulk_smem_bytes(bs);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gather_bulk_kernel, kBulkThreads, smem) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    const int64_t nbatch = (p->num_tokens + bs.rows - 1) / bs.rows;
    const int grid = (int)std::min<int64_t>(nbatch, (int64_t)per_sm * di.sms);
    gather_bulk_kernel<<<grid, kBulkThreads, smem, st>>>(a, bs);
    return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
  }
  // Otherwise (unaligned rows, or the QMLA_GATHER_REGS test hook): register-staged loads, a
  // persistent grid of resident blocks, each warp striding over groups of kGatherBatch rows.
  auto kern = vec ? gather_cache_kernel<true> : gather_cache_kernel<false>;
  static std::atomic<int> resident[2];  // blocks per SM of each variant, queried once
  int per_sm = resident[vec].load(std::memory_order_relaxed);
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 32 * kGatherWarps, 0) !=
            cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
    resident[vec].store(per_sm, std::memory_order_relaxed);
  }
  const int64_t rows_per_block = (int64_t)kGatherWarps * kGatherBatch;
  const int64_t blocks = (p->num_tokens + rows_per_block - 1) / rows_per_block;
  const int grid = (int)std::min<int64_t>(blocks, (int64_t)per_sm * di.sms);
  kern<<<grid, 32 * kGatherWarps, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? QMLA_OK : QMLA_E_CUDA;
}

}  // extern "C"
