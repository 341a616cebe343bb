// Paged latent-KV MLA decode for B200 (sm_100a).
//
// One persistent CTA per SM walks a balanced, contiguous range of 128-token
// tiles over all decode rows (rows are cut into segments at CTA boundaries and
// merged afterwards).  Warp roles (16 warps, 512 threads):
//   warps 0-7   softmax / epilogue.  Warp w reads TMEM sub-partition w%4 (tokens
//               32*(w%4) .. +31 of the tile, one token per lane) and owns half of
//               the heads (w/4)
//   warp  8     K loads: TMA boxes (two 128-byte columns x a run of tokens of one
//               page) into the K ring; warp 9 stages the rms tail.  Page sizes that
//               are not multiples of 16 use 16-byte cp.async gathers from warps 8-10
//   warps 10, 11, 15  V loads: re-read the tile's latent columns (L2-resident by then)
//               into the V ring once QK of the tile has finished.  One-column bf16 K slots:
//               warp 10 alone, one TMA box per 16 tokens carrying every column of the slot's
//               output blocks.  Otherwise 16-byte cp.async copies: with paired K slots
//               warps 10, 11 and 15 fill whole slots in turn, else two warps share each slot
//   warps 12-13 QK issuers (tcgen05), one S partial each; warp 12 owns TMEM
//   warp  14    PV issuer (tcgen05): per V slot, one MMA into each of the slot's
//               128-dim output blocks (two for e4m3: P's hi and lo terms); narrow MMAs
//               measured ~43 cycles each whether they hit one accumulator or rotate
// Per 128-token tile:
//   S^T[128 tok, heads] = K_tile . Q^T     tcgen05 M=128, K-major A and B
//   softmax over tokens with the per-(token, head) rms divisor, base 2, lazy
//   rescale (O is only rescaled when a running max grows by more than 2^8)
//   O^T[rank, heads]   += V^T . P^T        tcgen05 M=128, MN-major A and B
// K ring slot: 128 tokens x two 128-byte column chunks (32 KB), laid out as
// [8-token group][chunk][token in group][128 B], 128-byte swizzled.  Chunk c of a slot
// is then a K-major SW128 MMA operand that starts at c * 1 KB with its 8-row groups
// 2 KB apart, and one 5-D TMA box fills both chunks of a page run (4 KB for 16-token
// pages).  TMA moves ~1.5x more bytes per SM with these boxes than with 2 KB boxes of
// one column (probe: 46.9 vs 31.0 GB/s per SM), and 2 KB was the largest one-column
// box a 16-token page allows.  A slot holding the row's partial last chunk is loaded
// chunk by chunk through a 3-D map whose row extent zero-fills the columns past the
// QK width, and keeps the plain layout (chunk c's 128 rows contiguous at c * 16 KB).
// The tile is 128 tokens because one tcgen05.mma costs about the same issue time
// for M=64 and M=128 at these narrow N (24-48 heads): M=128 halves the QK MMAs per
// token, which bounded the 64-token design.  K slots are freed as soon as their QK
// MMAs complete, so the HBM stream never waits for the softmax.  bf16 caches use
// kind::f16.  FP8 caches use kind::f8f6f4 on the raw e4m3 tile; q and P are each
// split into two e4m3 terms (hi + lo): q's terms are stacked along N of the QK MMA
// (summed by the softmax), P's terms are two PV MMAs into the same accumulator.
// That keeps ~bf16 precision without a dequantisation pass over the cache.
// Semantics follow the reference Triton kernel
// qwen_mla/ops/mla_decode_attention.py:297-586 and its split merge :1064-1137.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "qmla_ptx.cuh"

namespace qmla {

constexpr int kTile = 128;         // tokens per tile (the QK MMA's M)
constexpr int kMaxQkChunks = 32;   // QK width <= 2048 bf16 elements (4 KB)
constexpr int kMaxCtas = 160;      // persistent CTAs per launch (B200: 148 SMs)
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kWarpK = 8, kNumKWarps = 3, kWarpV = 11, kWarpQK = 12, kWarpPV = 14;
constexpr int kWarpVX = 15;  // the extra V-load warp
constexpr int kNumWarps = 16, kNumThreads = kNumWarps * 32;
constexpr int kKThreads = kNumKWarps * 32;
constexpr int kRmsMaxUnits = 5;    // staged 16-byte units per token: <= 64 rms bytes + alignment
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P may reach 2^8 before O is rescaled
constexpr int kBarSoftmax = 1;             // named barrier id of the softmax warps
constexpr int kBarK = 2;                   // named barrier id of the K-load warps
constexpr int kKdoneDepth = 8;
constexpr int kEarlyQTiles = 16;           // segments this short stage the next Q early
// Register split of the widest shapes (32 or more query rows): the softmax warpgroups hold a
// running max, sum and scale per query row (NQK / 2 of each per thread), more than the 128
// registers a 512-thread CTA gives every thread; the loader / issuer warpgroups need far fewer.
// (kRegsSoftmax + kRegsProducer) * 256 threads = 128 * 512: the whole launch pool, no more.
constexpr uint32_t kRegsSoftmax = 184, kRegsProducer = 72;
constexpr int kRegsAtLaunch = 128;
// Tiles of a row bulk-prefetched into L2 ahead of the K loads (TMA mode).  Off: the
// prefetches share the bulk-copy engine with the K boxes and evicted the latent lines
// that the V loads re-read (DRAM bytes per launch rose from 1.07x to 1.47x of the
// algorithmic bytes on config 1 and throughput fell 8%).
#ifndef QMLA_PREFETCH_TILES
#define QMLA_PREFETCH_TILES 0
#endif
constexpr int kPrefetchTiles = QMLA_PREFETCH_TILES;

struct DecodeArgs {
  // query
  const uint8_t* q;
  const uint8_t* q_pe;
  int64_t q_sr, q_sh, qpe_sr, qpe_sh;  // element strides
  int q_dtype;
  int q_vec, qpe_vec;  // 16-byte vector loads are legal for q / q_pe rows
  // cache / paging
  const uint8_t* cache;
  int64_t page_stride_b, token_stride_b, num_pages;
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* seq_lens;
  int page_size;
  int use_tma;   // 1: K tiles by TMA boxes of run_rows tokens (page_size % 16 == 0)
  int run_rows;  // tokens per TMA box: gcd(page_size, 128)
  // geometry.  A work row is `fold` consecutive decode rows (MTP drafts of one request, which
  // share its block-table row) decoded together as R = fold * H query rows, so the request's
  // cache is read once per work row instead of once per draft.
  int num_rows;     // work rows (decode rows / fold)
  int fold, R;      // decode rows per work row; query rows per work row (fold * H)
  int H, rank, qk_dim, rms_mode;
  int qk_bytes;     // bytes of a cache row the QK contraction reads
  int row_bytes;    // bytes of a cache row (kv_row_width * element size)
  int n_qk_slots;   // K-ring slots loaded per tile (two 128-byte column chunks per slot)
  int n_sub_qk;     // 128-byte-wide MMA sub-chunks of the QK width
  int n_full_chunks;  // chunks that lie entirely inside the QK width
  int seg_cost;       // work-partition cost of a row's segment overhead, in tiles
  int early_q;        // segments of at most this many tiles stage the next segment's Q early
  int rms_base_b;   // 16-byte-aligned first byte of the rms tail in a row
  int rms_units;    // 16-byte units staged per token (0: no rms); staging stride = 16 * rms_units
  int rms_skip;     // first rms byte within the staged units
  int pf_bytes;     // bytes of a cache row prefetched into L2 (QK columns + rms tail)
  float sm_scale;
  float logit_cap;
  const float* k_scale;
  // outputs
  uint8_t* o;
  int64_t o_sr, o_sh;
  int o_dtype;
  uint8_t* lse;
  int64_t lse_sr;
  int lse_dtype;
  // workspace
  int* status;
  const int32_t* tile_prefix;   // [num_rows + 1]
  const int32_t* range_bounds;  // [G + 1] first tile of each CTA range (range_bound)
  const uint8_t* q_img;        // FP8: per work row, the Q buffer's shared-memory image (e4m3 hi/lo)
  const float* q_scale;        // FP8: per work row, NQK per-row q scales (448 / max|q|)
  int q_img_bytes;             // bytes of one image (the Q buffer)
  float* part_o;               // [2*G][R][rank]
  float* part_lse;             // [2*G][R] (log2 units)
  int* row_done;               // [num_rows] pieces written per work row (in-kernel merge), or null
  int G;
  // shared-memory layout (byte offsets from the 1024-aligned base)
  uint32_t off_kring, nk, off_vring, nv, off_q, q_chunk_bytes, off_p, p_bytes, off_rms, off_misc;
  int v_tma;              // 1: V slots by TMA boxes (needs use_tma); 0: by 16-byte cp.async
  int v_blocks;           // V by TMA: 128-dim output blocks per V slot (a divisor of rank / 128)
  uint32_t v_slot_bytes;  // V by TMA: bytes of a V slot (4 KB per output block)
  // Optional stage timestamps of CTA 0 (builds with -DQMLA_TRACE only):
  // trace[tile * 16 + event] = %globaltimer in ns.
  unsigned long long* trace;
  unsigned trace_cta;  // the CTA whose stages are traced
  int trace_tid;       // the softmax thread whose stages are traced
};

#ifdef QMLA_TRACE
#define QMLA_TR(ev)                                                                            \
  do {                                                                                         \
    if (a.trace && blockIdx.x == a.trace_cta && jt < 256) a.trace[jt * 16 + (ev)] = globaltimer_ns(); \
  } while (0)
#define QMLA_TRS(plane, idx)                                                     \
  do {                                                                           \
    if (a.trace && blockIdx.x == a.trace_cta && jt < 256)                        \
      a.trace[(plane) * 4096 + jt * 16 + (idx)] = globaltimer_ns();              \
  } while (0)
#else
#define QMLA_TR(ev) \
  do {              \
  } while (0)
#define QMLA_TRS(plane, idx) \
  do {                       \
  } while (0)
#endif

// ---------------------------------------------------------------- small helpers
__device__ __forceinline__ float load_as_float(const uint8_t* p, int dt) {
  if (dt == 0) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  if (dt == 1) return __half2float(*reinterpret_cast<const __half*>(p));
  return *reinterpret_cast<const float*>(p);
}
__device__ __forceinline__ void store_from_float(uint8_t* p, int dt, float v) {
  if (dt == 0)
    *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(v);
  else if (dt == 1)
    *reinterpret_cast<__half*>(p) = __float2half_rn(v);
  else
    *reinterpret_cast<float*>(p) = v;
}
__device__ __forceinline__ int dt_size(int dt) { return dt == 2 ? 4 : 2; }
__device__ __forceinline__ uint8_t f32_to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// Tokens of work row g: the longest of its decode rows (lengths < 0 count as 0); each query
// row masks the tokens past its own decode row's length.
__device__ __forceinline__ int work_len(const int32_t* seq_lens, int fold, int g) {
  int L = 0;
  for (int d = 0; d < fold; ++d) L = max(L, __ldg(seq_lens + (int64_t)g * fold + d));
  return L;
}
// Block-table row of work row g (its first decode row's: the drafts of a request share it).
__device__ __forceinline__ const int32_t* work_bt(const DecodeArgs& a, int g) {
  return a.block_table + (int64_t)g * a.fold * a.bt_stride;
}

// Segment iterator: the CTA's tile range [lo, hi) cut at row boundaries.
struct SegCursor {
  int row, lo, hi;
};
__device__ __forceinline__ int first_row_at(const int32_t* prefix, int n, int t) {
  int a = 0, b = n;  // invariant: prefix[a] <= t < prefix[b]
  while (b - a > 1) {
    int m = (a + b) >> 1;
    if (__ldg(prefix + m) <= t)
      a = m;
    else
      b = m;
  }
  return a;
}
__device__ __forceinline__ bool next_segment(const int32_t* prefix, SegCursor& c, int& row,
                                             int& k0, int& k1, int& p_lo, int& p_hi) {
  if (c.lo >= c.hi) return false;
  while (__ldg(prefix + c.row + 1) <= c.lo) ++c.row;
  row = c.row;
  p_lo = __ldg(prefix + row);
  p_hi = __ldg(prefix + row + 1);
  k0 = c.lo - p_lo;
  int end = p_hi < c.hi ? p_hi : c.hi;
  k1 = end - p_lo;
  c.lo = end;
  ++c.row;
  return true;
}

// First tile of CTA range c (c = 0..G; range c is [bound(c), bound(c+1))).  The tiles are
// split so that every CTA gets an equal share of the cost tiles + seg_cost * rows: a row's
// segment overhead (Q staging, pipeline refill, epilogue) counts as seg_cost tiles at its
// start.  A boundary that falls inside that overhead maps to the row's first tile, so a
// range can be empty.  Depends only on the lengths: the partition, and with it every
// reduction order, is the same for the same inputs.
// Plain loads: the plan kernel calls it on the prefix it has just written.
__device__ __forceinline__ int range_bound(const int32_t* prefix, int n, int G, int seg_cost, int c) {
  const int T = prefix[n];
  if (c <= 0) return 0;
  if (c >= G) return T;
  const int64_t C = (int64_t)T + (int64_t)seg_cost * n;
  const int64_t x = C * c / G;
  int lo = 0, hi = n;  // cost(lo) <= x < cost(hi), cost(r) = prefix[r] + seg_cost * r
  while (hi - lo > 1) {
    const int m = (lo + hi) >> 1;
    if ((int64_t)prefix[m] + (int64_t)seg_cost * m <= x)
      lo = m;
    else
      hi = m;
  }
  const int p0 = prefix[lo], p1 = prefix[lo + 1];
  int64_t off = x - ((int64_t)p0 + (int64_t)seg_cost * lo) - seg_cost;
  off = off < 0 ? 0 : off;
  off = off > (int64_t)(p1 - p0) ? (int64_t)(p1 - p0) : off;
  return p0 + (int)off;
}

// Row of the segment next_segment() would return next, or -1 (the cursor is not moved).
__device__ __forceinline__ int peek_segment_row(const int32_t* prefix, const SegCursor& c) {
  if (c.lo >= c.hi) return -1;
  int r = c.row;
  while (__ldg(prefix + r + 1) <= c.lo) ++r;
  return r;
}

// Address of 16-byte unit u of row r in a 128-byte-swizzled block (1024-aligned base).
__device__ __forceinline__ uint32_t sw128(uint32_t base, int r, int u) {
  return base + (uint32_t)(r * 128 + ((u ^ (r & 7)) << 4));
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z,
                                             uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
__device__ __forceinline__ void st_shared_v2(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t a) {
  uint32_t x;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(x) : "r"(a));
  return x;
}
__device__ __forceinline__ uint32_t ld_shared_u8(uint32_t a) {
  uint32_t x;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(x) : "r"(a));
  return x;
}
__device__ __forceinline__ void st_shared_u32(uint32_t a, uint32_t x) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(x) : "memory");
}

// Load N (4, 8, 12, 16 or 24) consecutive 32-bit columns of this thread's TMEM lane.
template <int N>
__device__ __forceinline__ void load_cols(uint32_t taddr, float* v) {
  if constexpr (N == 24) {
    tmem_ld16(taddr, v);
    tmem_ld8(taddr + 16, v + 16);
  } else if constexpr (N == 16) {
    tmem_ld16(taddr, v);
  } else if constexpr (N == 12) {
    tmem_ld8(taddr, v);
    tmem_ld4(taddr + 8, v + 8);
  } else if constexpr (N == 8) {
    tmem_ld8(taddr, v);
  } else {
    static_assert(N == 4, "4, 8, 12 or 16 columns");
    tmem_ld4(taddr, v);
  }
}

// Slot index and phase bit of a sequentially used mbarrier ring.
struct Ring {
  uint32_t idx = 0, ph = 0;
  __device__ __forceinline__ void next(uint32_t n) {
    if (++idx == n) {
      idx = 0;
      ph ^= 1;
    }
  }
};

// Cache-row address of token t (0..127) of tile k of a row; 0 past the row end
// or for a page id outside the cache (those rows are zero-filled, never read).
__device__ __forceinline__ uint64_t token_row_addr(const DecodeArgs& a, const int32_t* bt, int L,
                                                   int k, int t) {
  const int tok = k * kTile + t;
  if (tok >= L) return 0ull;
  const int pg = __ldg(bt + tok / a.page_size);
  if (pg < 0 || pg >= a.num_pages) return 0ull;
  return reinterpret_cast<uint64_t>(a.cache + (int64_t)pg * a.page_stride_b +
                                    (int64_t)(tok % a.page_size) * a.token_stride_b);
}

// Tensor maps over the paged cache (TMA mode).
//   chunk: 3-D (row element, token in page, page); box = one 128-byte column x run tokens.
//          Its row extent is the QK width, so columns past it are zero-filled.
//   pair:  5-D (element of a 128-byte column, token in an 8-token group, column,
//          8-token group in the page, page); box = two columns x run tokens, landing in
//          the paired slot layout.  Its column extent counts only full columns.
//   vrows: the pair map's 5-D view with box = v_blocks output blocks (their 128-byte
//          columns) x 16 tokens, landing as [8-token group][column][token][128 B]: the V
//          slot layout the PV MMA reads directly.
// Pages outside [0, num_pages) are zero-filled by all three.
struct CacheMaps {
  CUtensorMap chunk;
  CUtensorMap pair;
  CUtensorMap vrows;
};

// With paired slots (PAIR), K slot s uses the plain layout (loaded column by column
// through the 3-D map) when it holds a column that extends past the QK width (TMA mode);
// otherwise the paired layout.  Without PAIR every slot holds one column, plain.
template <bool PAIR>
__device__ __forceinline__ bool slot_plain(const DecodeArgs& a, int s) {
  if constexpr (!PAIR) {
    return true;
  } else {
    const int last = min(2 * s + 1, a.n_sub_qk - 1);
    return a.use_tma && last >= a.n_full_chunks;
  }
}

// ---------------------------------------------------------------- the kernel
// PAIR: K slots of two columns (paired layout, 4 KB TMA boxes), chosen for rank 768 with up to
// 32 query rows.  Otherwise one column per K slot.
template <bool FP8, int NB, int NQK, bool PAIR>
__global__ void __launch_bounds__(kNumThreads, 1)
    mla_decode_kernel(const __grid_constant__ CacheMaps maps, const DecodeArgs a) {
  static_assert(NQK % 8 == 0 && NQK >= 8 && NQK <= 48, "query rows rounded to 8..48");
  constexpr int NPV = NQK <= 16 ? 16 : NQK <= 32 ? 32 : 48;  // PV MMA N (multiple of 16)
  // QK MMA N: heads rounded up to 16 for bf16 (the extra B rows are read from the next Q
  // chunk and only produce S columns nobody reads); the hi|lo q rows for FP8.
  constexpr int NQKM = FP8 ? 2 * NQK : NPV;
  // K ring slot: 128 tokens x two 128-byte column chunks of the row (the layout is in the
  // file header).  V ring slot, TMA mode: kVTokT tokens (one PV K step) x v_blocks output
  // blocks, [8-token group][column][token][128 B]; cp.async mode: 64 tokens x one block.
  constexpr int kKChunkBytes = 16384;             // one column chunk of 128 tokens
  constexpr int CPS = PAIR ? 2 : 1;               // column chunks per K slot
  constexpr uint32_t kKSlotBytes = kKChunkBytes * CPS;
  // V by TMA boxes: built into the bf16 one-column-K kernels only (the planner's choice there);
  // the other kernels keep only the cp.async fills.
  constexpr bool kVBoxes = !FP8 && !PAIR;
  constexpr int kCpb = FP8 ? 1 : 2;               // 128-byte columns per 128-dim output block
  constexpr int kVTokT = FP8 ? 32 : 16;           // tokens per V slot (TMA mode)
  constexpr int kVStepsT = kTile / kVTokT;        // token steps per tile (TMA mode)
  constexpr int VG = PAIR ? 3 : 1;                // V slot groups when V is copied (see the V loader)
  constexpr int kVSlotBytes = FP8 ? 8192 : 16384;  // cp.async mode
  constexpr int kVUnits = (FP8 ? 1 : 2) * 8;      // 16-byte units per token per V slot
  constexpr int kVTok = 64;                       // tokens per V slot (cp.async mode)
  constexpr int OW = NPV;                         // TMEM columns per O block
  constexpr int SWP = FP8 ? 2 * NPV : NPV;        // TMEM columns per S partial (hi|lo for FP8)
  // S partials: one per QK issuer (two issuers, each every other K step, when TMEM holds two
  // double-buffered partials next to O); the widest FP8 shapes (48 query rows, hi | lo: 96
  // columns per partial) keep one issuer and one partial so that S stays double-buffered (QK of
  // tile k+1 overlaps the softmax of tile k): O 6 x 48 + S 2 x 96 = 480 of 512 columns.  A single
  // S buffer with two partials measured 1.28x slower on config 2.
  constexpr int KP = (NB * OW + 2 * 2 * SWP <= 512) ? 2 : 1;
  constexpr int SW = KP * SWP;                    // TMEM columns per S buffer
  constexpr int SB = (NB * OW + 2 * SW <= 512) ? 2 : 1;  // S buffers
  constexpr uint32_t kCols = NB * OW + SB * SW;
  constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                 : kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "TMEM budget");
  constexpr int NJ = NQK / 2;   // heads per softmax thread (one token, half of the heads)
  constexpr int NH = NPV / 2;   // P^T / O^T columns per head half (NJ real + zero padding)
  constexpr int kPvSteps = FP8 ? 2 : 4;  // K = 32 (e4m3) or 16 (bf16) tokens per PV MMA
  constexpr int kPvAStep = FP8 ? 4096 : 2048;
  constexpr int kPvBStep = (FP8 ? 4 : 2) * 16 * NPV;
  constexpr int kPvHalfB = (kVTok / 8) * 16 * NPV;  // P^T bytes of one V slot's tokens

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ------------------------------------------------ work range
  const int total = __ldg(a.tile_prefix + a.num_rows);
  const int range_lo = __ldg(a.range_bounds + blockIdx.x);
  const int range_hi = __ldg(a.range_bounds + blockIdx.x + 1);
  (void)total;
  if (a.row_done) {
    // in-kernel merge mode (no merge kernel follows): work rows without tokens get o = 0 and
    // lse = -inf here, row r by CTA r % G
    for (int r = blockIdx.x; r < a.num_rows; r += gridDim.x) {
      if (__ldg(a.tile_prefix + r + 1) != __ldg(a.tile_prefix + r)) continue;
      const int osz = dt_size(a.o_dtype);
      for (int i = threadIdx.x; i < a.R * a.rank; i += blockDim.x) {
        const int q = i / a.rank, d = i - q * a.rank, dq = q / a.H;
        store_from_float(a.o + (((int64_t)r * a.fold + dq) * a.o_sr + (int64_t)(q - dq * a.H) * a.o_sh + d) * osz,
                         a.o_dtype, 0.f);
      }
      if (a.lse)
        for (int q = threadIdx.x; q < a.R; q += blockDim.x) {
          const int dq = q / a.H;
          store_from_float(a.lse + (((int64_t)r * a.fold + dq) * a.lse_sr + (q - dq * a.H)) * dt_size(a.lse_dtype),
                           a.lse_dtype, -INFINITY);
        }
    }
  }
  if (range_lo >= range_hi) return;  // uniform for the whole CTA
  const int row0 = first_row_at(a.tile_prefix, a.num_rows, range_lo);
#ifdef QMLA_TRACE
  if (a.trace && threadIdx.x == 0) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    a.trace[6 * 4096 + blockIdx.x * 2] = globaltimer_ns();
    a.trace[6 * 4096 + 2048 + blockIdx.x] = smid;
  }
#endif

  // ------------------------------------------------ barriers and scratch
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_misc);
  const uint32_t nk = a.nk, nv = a.nv;
  const uint32_t b_kfull = 0;                    // [nk] K slot landed (cp.async arrivals)
  const uint32_t b_kempty = nk;                  // [nk] K slot free (both QK issuers)
  const uint32_t b_vfull = 2 * nk;               // [nv] V slot landed
  const uint32_t b_vempty = 2 * nk + nv;         // [nv] V slot free
  const uint32_t b_sfull = 2 * (nk + nv);        // [2] S ready (both QK issuers)
  const uint32_t b_sempty = b_sfull + 2;         // [2] S consumed
  const uint32_t b_pfull = b_sempty + 2;         // [2] P written (+ O rescaled)
  const uint32_t b_odone = b_pfull + 2;          // [2] PV finished
  const uint32_t b_rfull = b_odone + 2;          // [2] rms tail staged
  const uint32_t b_rempty = b_rfull + 2;         // [2] rms staging consumed
  const uint32_t b_qfull = b_rempty + 2;         // [1] Q staged
  const uint32_t b_ofree = b_qfull + 1;          // [1] O read by the epilogue
  const uint32_t b_kdone = b_ofree + 1;          // [kKdoneDepth] QK of a tile finished
  const uint32_t b_fin = b_kdone + kKdoneDepth;  // [4] issuer drain at teardown
  const uint32_t n_bars = b_fin + 4;
  auto bar = [&](uint32_t i) -> uint32_t { return smem_u32(bars + i); };
  uint8_t* misc2 = smem + a.off_misc + ((n_bars * 8 + 15) / 16) * 16;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc2 + 4);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(misc2 + 8);  // in-kernel merge: this CTA is last
  float* red = reinterpret_cast<float*>(misc2 + 16);  // [2 halves][4 sp][32]
  float* hv = red + 256;                              // [4][64] per-query-row broadcast values
  // hv[0..63] alpha, hv[64..127] l, hv[128..191] m, hv[192..255] q scale (FP8)
  uint64_t* tokptr = reinterpret_cast<uint64_t*>(hv + 256);  // [2][128] K-load row addresses

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nk; ++i) {
      mbar_init(bar(b_kfull + i), a.use_tma ? 1 : kKThreads);
      mbar_init(bar(b_kempty + i), KP);
    }
    for (uint32_t i = 0; i < nv; ++i) {
      mbar_init(bar(b_vfull + i), (kVBoxes && a.v_tma) ? 1 : VG == 3 ? 32 : 64);  // one TMA arm, or the copying warps
      mbar_init(bar(b_vempty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(b_sfull + i), KP);
      mbar_init(bar(b_sempty + i), kSoftmaxWarps);
      mbar_init(bar(b_pfull + i), kSoftmaxWarps);
      mbar_init(bar(b_odone + i), 1);
      mbar_init(bar(b_rfull + i), a.use_tma ? 32 : kKThreads);
      mbar_init(bar(b_rempty + i), kSoftmaxWarps);
    }
    for (int i = 0; i < kKdoneDepth; ++i) mbar_init(bar(b_kdone + i), KP);
    for (int i = 0; i < 4; ++i) mbar_init(bar(b_fin + i), 1);
    mbar_init(bar(b_qfull), kSoftmaxWarps);
    mbar_init(bar(b_ofree), kSoftmaxWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpQK) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  static_assert((kRegsSoftmax + kRegsProducer) * 256 <= kRegsAtLaunch * kNumThreads, "register pool");
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t col_o = 0;
  const uint32_t col_s = NB * OW;

  const uint32_t kring = sbase + a.off_kring;
  const uint32_t vring = sbase + a.off_vring;
  const uint32_t qbuf = sbase + a.off_q;
  const uint32_t pbuf = sbase + a.off_p;
  const uint32_t rmsbuf = sbase + a.off_rms;  // [2][128 tokens][rstride]
  const int rstride = 16 * a.rms_units;       // rms staging bytes per token
  int* status = a.status;

  // Roles, one branch per warpgroup at the top so each warpgroup's register budget
  // (setmaxnreg, same instruction for its four warps) governs all of its code.
  if (warp >= kSoftmaxWarps) {
  if constexpr (NQK >= 32) setmaxnreg_dec<kRegsProducer>();
  if (a.use_tma && warp == kWarpK) {
    // ====================================================== K loads by TMA
    // Per slot: one paired box per run of tokens within a page (both columns at once),
    // or, for a slot with the partial last column, one 3-D box per (column, run); lanes
    // issue the boxes of a slot side by side.
    const uint64_t pol_lat = policy_evict_normal();
    const uint64_t pol_rope = policy_evict_first();
    const int run = a.run_rows, nrun = kTile / run;
    const int xstep = FP8 ? 128 : 64;  // column width in elements
    const int lat_chunks = a.rank * (FP8 ? 1 : 2) / 128;  // columns the V loads read again
    if (lane == 0) {
      prefetch_tmap(&maps.chunk);
      prefetch_tmap(&maps.pair);
    }
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, armed = 0;
    Ring r;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      const int L = work_len(a.seq_lens, a.fold, row);
      const int32_t* bt = work_bt(a, row);
      // page of token run `lane` of a tile (-1: past the row end, loads zeros)
      auto run_page = [&](int k) -> int {
        const int tok = k * kTile + lane * run;
        return (lane < nrun && tok < L) ? __ldg(bt + tok / a.page_size) : -1;
      };
      int pg = run_page(k0);
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        // this lane's box in a plain slot: column lane / nrun, token run lane % nrun; in
        // a paired slot: token run lane
        const int bg = lane % nrun, bc = lane / nrun;
        const int mypg = __shfl_sync(0xffffffffu, pg, bg);
        const int y = (k * kTile + bg * run) % a.page_size;
        int pg_next = -1;  // the next tile's page ids load while this tile's slots issue
        for (int s = 0; s < a.n_qk_slots && ok; ++s) {
          if (s == 0 && k + 1 < k1) pg_next = run_page(k + 1);
          const bool plain = slot_plain<PAIR>(a, s);
          const int c0 = CPS * s;  // first column chunk of the slot
          const int nch = min(CPS, a.n_sub_qk - c0);
          if (lane == 0) {
            ok = mbar_wait(bar(b_kempty + r.idx), r.ph ^ 1, abort_flag, status);
            if (ok)
              mbar_expect_tx(bar(b_kfull + r.idx),
                             plain ? (uint32_t)(nch * kKChunkBytes) : kKSlotBytes);
            QMLA_TRS(4, s);
            if (s == 0) QMLA_TR(0);
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (ok) {
            const uint32_t slot = kring + r.idx * kKSlotBytes;
            if (plain) {
              if (lane < nch * nrun)
                tma_load_3d(slot + bc * kKChunkBytes + bg * run * 128, &maps.chunk,
                            (c0 + bc) * xstep, y, mypg, bar(b_kfull + r.idx),
                            c0 + bc < lat_chunks ? pol_lat : pol_rope);
            } else if (lane < nrun) {
              tma_load_5d(slot + lane * run * 256, &maps.pair, 0, 0, c0, y / 8, mypg,
                          bar(b_kfull + r.idx), c0 < lat_chunks ? pol_lat : pol_rope);
            }
            ++armed;
          }
          if (lane == 0) QMLA_TRS(1, s);
          r.next(nk);
        }
        pg = pg_next;
      }
    }
    // After an abort: wait (bounded) for the boxes already issued, so no copy still
    // targets this CTA's shared memory when it exits.
    if (!ok && lane == 0) {
      for (uint32_t p = armed > nk ? armed - nk : 0u; p < armed; ++p) {
        volatile int never = 0;
        mbar_wait(bar(b_kfull + p % nk), (p / nk) & 1, &never, nullptr, 20000000ull);
      }
    }
    __syncwarp();
  } else if (a.use_tma && warp == kWarpK + 1) {
    // ====================================================== rms tail + L2 prefetch (TMA mode)
    // One warp; lane handles tokens lane + 32 * i (i < 4) of each tile.
    const uint64_t pol_lat = policy_evict_normal();
    const uint64_t pol_rope = policy_evict_first();
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      const int L = work_len(a.seq_lens, a.fold, row);
      const int32_t* bt = work_bt(a, row);
      for (int kp = k0; kp < min(k1, k0 + kPrefetchTiles); ++kp) {  // no-op unless enabled
        for (int h2 = 0; h2 < kTile / 32; ++h2) {
          const uint64_t pa = token_row_addr(a, bt, L, kp, lane + 32 * h2);
          if (pa) bulk_prefetch_l2(reinterpret_cast<const void*>(pa), a.pf_bytes, pol_lat);
        }
      }
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        if (kPrefetchTiles > 0 && k + kPrefetchTiles < k1) {
          for (int h2 = 0; h2 < kTile / 32; ++h2) {
            const uint64_t pa = token_row_addr(a, bt, L, k + kPrefetchTiles, lane + 32 * h2);
            if (pa) bulk_prefetch_l2(reinterpret_cast<const void*>(pa), a.pf_bytes, pol_lat);
          }
        }
        if (a.rms_units > 0) {
          const uint32_t tb = jt & 1;
          if (jt >= 2) ok = mbar_wait(bar(b_rempty + tb), ((jt - 2) >> 1) & 1, abort_flag, status);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            for (int h2 = 0; h2 < kTile / 32; ++h2) {
              const int t = lane + 32 * h2;
              const uint64_t src = token_row_addr(a, bt, L, k, t);
              for (int u = 0; u < a.rms_units; ++u) {
                const int col = a.rms_base_b + 16 * u;
                const int nbytes = src ? max(0, min(16, a.row_bytes - col)) : 0;
                cp_async_16_hint(rmsbuf + tb * (kTile * rstride) + t * rstride + 16 * u,
                                 nbytes ? reinterpret_cast<const void*>(src + col) : a.cache,
                                 (uint32_t)nbytes, pol_rope);
              }
            }
            cp_async_mbar_arrive(bar(b_rfull + tb));
          }
        }
      }
    }
    if (!ok) asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (!a.use_tma && warp >= kWarpK && warp < kWarpK + kNumKWarps) {
    // ====================================================== K loads by cp.async (+ rms tail)
    const int pt = threadIdx.x - kWarpK * 32;  // 0..95
    const uint64_t pol_lat = policy_evict_normal();  // latent columns: read again for PV
    const uint64_t pol_rope = policy_evict_first();  // rope columns: read once
    const int lat_chunks = a.rank * (FP8 ? 1 : 2) / 128;
    // row addresses of tokens pt and pt + 96 of a tile (the tile's 128 tokens)
    const int t1 = pt + kKThreads < kTile ? pt + kKThreads : -1;
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0;
    Ring r;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      const int L = work_len(a.seq_lens, a.fold, row);
      const int32_t* bt = work_bt(a, row);
      uint64_t nptr0 = token_row_addr(a, bt, L, k0, pt);
      uint64_t nptr1 = t1 >= 0 ? token_row_addr(a, bt, L, k0, t1) : 0ull;
      // optional L2 prefetch kPrefetchTiles ahead of the loads (off by default)
      for (int kp = k0; kp < min(k1, k0 + kPrefetchTiles); ++kp) {
        for (int h2 = 0; h2 < 2; ++h2) {
          const int t = h2 ? t1 : pt;
          const uint64_t pa = t < 0 ? 0ull : token_row_addr(a, bt, L, kp, t);
          if (pa) bulk_prefetch_l2(reinterpret_cast<const void*>(pa), a.pf_bytes, pol_lat);
        }
      }
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const uint32_t tb = jt & 1;
        tokptr[tb * kTile + pt] = nptr0;
        if (t1 >= 0) tokptr[tb * kTile + t1] = nptr1;
        named_bar_sync(kBarK, kKThreads);
        if (kPrefetchTiles > 0 && k + kPrefetchTiles < k1) {
          for (int h2 = 0; h2 < 2; ++h2) {
            const int t = h2 ? t1 : pt;
            const uint64_t pa = t < 0 ? 0ull : token_row_addr(a, bt, L, k + kPrefetchTiles, t);
            if (pa) bulk_prefetch_l2(reinterpret_cast<const void*>(pa), a.pf_bytes, pol_lat);
          }
        }
        if (k + 1 < k1) {  // the next tile's row addresses
          nptr0 = token_row_addr(a, bt, L, k + 1, pt);
          if (t1 >= 0) nptr1 = token_row_addr(a, bt, L, k + 1, t1);
        }
        const uint64_t* tp = tokptr + tb * kTile;
        // ---- rms tail of the tile -> staging buffer tb
        if (a.rms_units > 0) {
          if (jt >= 2) ok = mbar_wait(bar(b_rempty + tb), ((jt - 2) >> 1) & 1, abort_flag, status);
          if (ok) {
            for (int q = pt; q < kTile * a.rms_units; q += kKThreads) {
              const int t = q / a.rms_units, u = q - t * a.rms_units;
              const uint64_t src = tp[t];
              const int col = a.rms_base_b + 16 * u;
              const int nbytes = src ? max(0, min(16, a.row_bytes - col)) : 0;
              cp_async_16_hint(rmsbuf + tb * (kTile * rstride) + t * rstride + 16 * u,
                               nbytes ? reinterpret_cast<const void*>(src + col) : a.cache,
                               (uint32_t)nbytes, pol_rope);
            }
            cp_async_mbar_arrive(bar(b_rfull + tb));
          }
        }
        // ---- QK columns, two 128-byte column chunks per slot (paired layout); eight
        // consecutive threads copy the 128 bytes of one (token, chunk)
        for (int s = 0; s < a.n_qk_slots; ++s) {
          if (ok) ok = mbar_wait(bar(b_kempty + r.idx), r.ph ^ 1, abort_flag, status);
          if (pt == 0) QMLA_TRS(4, s);
          if (pt == 0 && s == 0) QMLA_TR(0);
          if (ok) {
            const uint32_t dst0 = kring + r.idx * kKSlotBytes;
            const int c0 = CPS * s;
            const int nch = min(CPS, a.n_sub_qk - c0);
            const bool plain = slot_plain<PAIR>(a, s);
            const int upt = 8 * nch;  // 16-byte units per token in this slot
            const uint64_t pol = c0 < lat_chunks ? pol_lat : pol_rope;
#pragma unroll 4
            for (int q = pt; q < kTile * upt; q += kKThreads) {
              const int t = q / upt, rem = q - t * upt, ci = rem >> 3, u = rem & 7;
              const int colb = (c0 + ci) * 128 + u * 16;              // byte column of the row
              const int nbytes = max(0, min(16, a.qk_bytes - colb));  // zero past the QK width
              const uint64_t src = tp[t];
              const uint32_t nb = src ? (uint32_t)nbytes : 0u;
              const uint32_t row = plain ? dst0 + ci * kKChunkBytes + t * 128
                                         : dst0 + (t >> 3) * 2048 + ci * 1024 + (t & 7) * 128;
              cp_async_16_hint(row + ((u ^ (t & 7)) << 4),
                               nb ? reinterpret_cast<const void*>(src + colb) : a.cache, nb, pol);
            }
            cp_async_mbar_arrive(bar(b_kfull + r.idx));
          }
          if (pt == 0) QMLA_TRS(1, s);
          if (pt == 0 && s == a.n_qk_slots - 1) QMLA_TR(1);
          r.next(nk);
        }
        // every K thread leaves the tile together (and tokptr[tb] is free again)
        ok = !named_bar_or(kBarK, kKThreads, !ok);
      }
    }
    if (!ok) asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (kVBoxes && a.v_tma && warp == kWarpK + 2) {
    // ====================================================== V loads by TMA (from L2)
    // Once QK(jt) has consumed the tile, its latent columns are in L2.  A V slot holds one PV
    // K step of tokens (32 e4m3 / 16 bf16) x v_blocks output blocks; one box per 16 tokens of
    // a page carries all of the slot's 128-byte columns (v_blocks x 2 or 4 KB), so a tile
    // takes 8 boxes per block group instead of a 16-byte copy per (token, column unit):
    // 16-byte cp.async fills ran at ~20 GB/s per SM, TMA boxes of 12-24 KB from L2 at
    // 115-133 GB/s.  Lanes 0-7 hold the page and 8-token group of the tile's 16-token runs.
    const uint64_t pol = policy_evict_first();  // the latent's last use in this call
    const int vb = a.v_blocks, nbg = NB / vb;
    const int cv = vb * kCpb;                   // 128-byte columns per slot row group
    constexpr int kBoxTok = 16;
    constexpr int kBoxes = kVTokT / kBoxTok;    // boxes per slot: 2 (e4m3) or 1 (bf16)
    const uint32_t box_bytes = (uint32_t)(kBoxTok * cv * 128);
    if (lane == 0) prefetch_tmap(&maps.vrows);
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, armed = 0;
    Ring r;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      const int L = work_len(a.seq_lens, a.fold, row);
      const int32_t* bt = work_bt(a, row);
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        int pg = -1, gy = 0;  // page (-1: past the row end, loads zeros) and 8-token group
        if (lane < kTile / kBoxTok) {
          const int tok = k * kTile + lane * kBoxTok;
          if (tok < L) {
            pg = __ldg(bt + tok / a.page_size);
            gy = (tok % a.page_size) / 8;
          }
        }
        if (lane == 0)
          ok = mbar_wait(bar(b_kdone + (jt % kKdoneDepth)), (jt / kKdoneDepth) & 1, abort_flag,
                         status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (lane == 0) QMLA_TR(6);
        for (int vs = 0; vs < kVStepsT * nbg && ok; ++vs) {  // token step vs / nbg, block group vs % nbg
          const int ts = vs / nbg, bg = vs - ts * nbg;
          // A 16-token run that straddles the row end would bring the page's stale rows past
          // L, and P = 0 times a NaN there is NaN: such a slot is copied 16 bytes per lane
          // instead, zero-filled past L (at most one slot per row).
          const int t0 = k * kTile + ts * kVTokT;
          const bool ragged = (L & 15) != 0 && L > t0 && L < t0 + kVTokT;
          const uint32_t slot = vring + r.idx * a.v_slot_bytes;
          if (lane == 0) {
            ok = mbar_wait(bar(b_vempty + r.idx), r.ph ^ 1, abort_flag, status);
            if (ok && !ragged) mbar_expect_tx(bar(b_vfull + r.idx), a.v_slot_bytes);
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (ok && !ragged) {
            const int run = ts * kBoxes + (lane < kBoxes ? lane : 0);
            const int mypg = __shfl_sync(0xffffffffu, pg, run);
            const int myg = __shfl_sync(0xffffffffu, gy, run);
            if (lane < kBoxes)
              tma_load_5d(slot + lane * box_bytes, &maps.vrows, 0, 0, bg * cv, myg, mypg,
                          bar(b_vfull + r.idx), pol);
            ++armed;
          } else if (ok) {
            // unit i: token i / (cv * 8) of the slot, column (i / 8) % cv, 16-byte unit i % 8,
            // at the slot layout's swizzled position
            for (int i = lane; i < kVTokT * cv * 8; i += 32) {
              const int tl = i / (cv * 8), rem = i - tl * (cv * 8), c = rem >> 3, u = rem & 7;
              const uint64_t src = token_row_addr(a, bt, L, k, ts * kVTokT + tl);
              const int colb = (bg * cv + c) * 128 + u * 16;
              cp_async_16_hint(slot + (uint32_t)((tl >> 3) * cv * 1024 + c * 1024 + (tl & 7) * 128 +
                                                 ((u ^ (tl & 7)) << 4)),
                               src ? reinterpret_cast<const void*>(src + colb) : a.cache,
                               src ? 16u : 0u, pol);
            }
            cp_async_mbar_arrive_extra(bar(b_vfull + r.idx));
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(b_vfull + r.idx));  // the slot's expected arrival
          }
          if (lane == 0 && vs < 16) QMLA_TRS(3, vs);
          r.next(nv);
        }
        if (lane == 0) QMLA_TR(13);
      }
    }
    // After an abort: wait (bounded) for the boxes already issued, and for the copies.
    if (!ok) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      if (lane == 0) {
        for (uint32_t p = armed > nv ? armed - nv : 0u; p < armed; ++p) {
          volatile int never = 0;
          mbar_wait(bar(b_vfull + p % nv), (p / nv) & 1, &never, nullptr, 20000000ull);
        }
      }
    }
    __syncwarp();
  } else if (!(kVBoxes && a.v_tma) && (warp == kWarpV || warp == kWarpVX || (a.use_tma && warp == kWarpK + 2))) {
    // ====================================================== V loads by cp.async (from L2)
    // (e4m3 caches and paired bf16 K slots: their K boxes would queue behind V boxes in the
    // SM's TMA unit; page sizes that rule TMA out)
    // V slot number n (counted over the CTA's whole run) is filled by group n % v_groups.
    // v_groups == 3 (TMA mode): warps 10, 11 and 15 each fill whole slots in turn (more
    // copies in flight; the config-1 shape gains).  v_groups == 1: warps 10 and 11 (TMA
    // mode) or 11 and 15 (cp.async mode) split the 64 tokens of every slot (lower latency
    // per slot; smaller heads/ranks gain).
    const uint64_t pol = policy_evict_first();
    constexpr int ngroups = VG;
    const int vi = warp == kWarpV ? 0 : warp == kWarpVX ? 1 : 2;  // 11, 15, 10
    constexpr int gw = VG == 3 ? 1 : 2;                            // warps per group
    const int vg = VG == 3 ? vi : 0;                               // this warp's group
    const int gi = VG == 3 ? 0 : (a.use_tma ? (warp == kWarpV ? 1 : 0) : vi);
    const bool active = VG == 3 || (a.use_tma ? warp != kWarpVX : true);
    constexpr int tpw = kVTok / gw;  // tokens of a V slot per warp of its group
    constexpr int kTokStep = 32 / kVUnits;  // tokens per warp-wide copy step
    uint32_t vseq = 0;  // V slots seen so far
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0;
    Ring r;
    bool ok = active;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      const int L = work_len(a.seq_lens, a.fold, row);
      const int32_t* bt = work_bt(a, row);
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        // this lane's tokens of V slot half hh: hh*64 + gi*tpw + lane (and + 32 when one
        // warp covers the slot)
        uint64_t ph[2][2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          ph[hh][0] = token_row_addr(a, bt, L, k, hh * kVTok + gi * tpw + lane);
          ph[hh][1] = tpw > 32 ? token_row_addr(a, bt, L, k, hh * kVTok + gi * tpw + lane + 32) : 0ull;
        }
        // the latent part is read again only after QK(jt) consumed it (it is in L2)
        ok = mbar_wait(bar(b_kdone + (jt % kKdoneDepth)), (jt / kKdoneDepth) & 1, abort_flag,
                       status);
        ok = __all_sync(0xffffffffu, ok);
        if (lane == 0 && vi == 0) QMLA_TR(6);
        for (int bh = 0; bh < 2 * NB && ok; ++bh, ++vseq) {  // block bh/2, token half bh%2
          const int b = bh >> 1, hh = bh & 1;
          if (ngroups > 1 && (int)(vseq % (uint32_t)ngroups) != vg) {  // another group's slot
            r.next(nv);
            continue;
          }
          ok = mbar_wait(bar(b_vempty + r.idx), r.ph ^ 1, abort_flag, status);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) {
            const uint32_t dst0 = vring + r.idx * kVSlotBytes;
            const int u = lane % kVUnits, sc = u >> 3, v = u & 7;
            const int colb = FP8 ? b * 128 + v * 16 : (b * 128 + sc * 64 + v * 8) * 2;
            const int steps = tpw / kTokStep;
            const uint64_t p0 = ph[hh][0], p1 = ph[hh][1];
#pragma unroll 8
            for (int i = 0; i < steps; ++i) {
              const int tl = i * kTokStep + lane / kVUnits;  // token within this warp's part
              const uint64_t src = __shfl_sync(0xffffffffu, i * kTokStep < 32 ? p0 : p1, tl & 31);
              const int t = gi * tpw + tl;  // token within the V slot
              cp_async_16_hint(dst0 + sc * 8192 + t * 128 + ((v ^ (t & 7)) << 4),
                               src ? reinterpret_cast<const void*>(src + colb) : a.cache,
                               src ? 16u : 0u, pol);
            }
            cp_async_mbar_arrive(bar(b_vfull + r.idx));
          }
          if (lane == 0 && bh < 16) QMLA_TRS(3, bh);
          r.next(nv);
        }
        if (lane == 0 && vi == 0) QMLA_TR(13);
      }
    }
    if (!ok) asm volatile("cp.async.wait_all;" ::: "memory");
  } else if (warp == kWarpQK || warp == kWarpQK + 1) {
    // ====================================================== QK issuers
    // With two S partials each warp issues every other 16/32-wide K step of every column
    // chunk into its own partial (the softmax sums them): one thread issuing all MMAs of a
    // tile was 10% slower overall for 24 heads.  With one partial (KP = 1) warp 12 issues all.
    const int qw = warp - kWarpQK;
    if (lane == 0 && qw < KP) {
      const uint32_t idesc = make_idesc_f16(FP8 ? 0 : 1, 128, NQKM, 0, 0);
      const uint32_t qc16 = a.q_chunk_bytes >> 4;              // Q chunk stride, descriptor units
      const uint64_t q_desc0 = make_sdesc(qbuf, 16, 1024, 2);  // Q chunk 0 (K-major, 128B swizzle)
      SegCursor cur{row0, range_lo, range_hi};
      int row, k0, k1, plo, phi;
      uint32_t jt = 0, sidx = 0;
      Ring r;
      bool ok = true;
      while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
        ok = mbar_wait(bar(b_qfull), sidx & 1, abort_flag, status);
        for (int k = k0; k < k1 && ok; ++k, ++jt) {
          const uint32_t sb = jt % SB;
          if (jt >= SB) ok = mbar_wait(bar(b_sempty + sb), ((jt - SB) / SB) & 1, abort_flag, status);
          if (qw == 0) QMLA_TR(2);
          tc_fence_after();
          const uint32_t d_s = tmem_base + col_s + sb * SW + qw * SWP;
          for (int s = 0; s < a.n_qk_slots && ok; ++s) {
            ok = mbar_wait(bar(b_kfull + r.idx), r.ph, abort_flag, status);
            if (!ok) break;
            if (qw == 0) QMLA_TRS(2, s);
            if (qw == 0 && s == 0) QMLA_TR(3);
            if (qw == 0 && s == a.n_qk_slots - 1) QMLA_TR(4);
            fence_proxy_async_smem();  // cp.async writes -> tensor-core reads
            tc_fence_after();
            // A = column chunk ci of the slot (M = 128 tokens, K-major, 128-byte swizzle):
            //   paired layout: starts at ci * 1 KB, 8-row groups 2 KB apart;
            //   plain layout:  starts at ci * 16 KB, 8-row groups 1 KB apart.
            // B = Q chunk 2s + ci (N rows, K-major SW128).  K step = 32 bytes.
            const bool plain = slot_plain<PAIR>(a, s);
            const int c0 = CPS * s;
            const int nch = min(CPS, a.n_sub_qk - c0);
            const uint32_t slot = kring + r.idx * kKSlotBytes;
#pragma unroll
            for (int ci = 0; ci < CPS; ++ci) {
              if (ci < nch) {
                const uint64_t ad0 = plain ? make_sdesc(slot + ci * kKChunkBytes, 16, 1024, 2)
                                           : make_sdesc(slot + ci * 1024, 16, 2048, 2);
                const uint64_t bd0 = q_desc0 + (uint64_t)(c0 + ci) * qc16;
#pragma unroll
                for (int kk = 0; kk < 4 / KP; ++kk) {  // 4 K steps of 32 bytes per column
                  const int ks = KP * kk + qw;
                  const uint32_t acc = (s == 0 && ci == 0 && kk == 0) ? 0u : 1u;
                  if constexpr (FP8)
                    tc_mma_f8_ss(d_s, ad0 + (uint64_t)(ks * 2), bd0 + (uint64_t)(ks * 2), idesc, acc);
                  else
                    tc_mma_f16_ss(d_s, ad0 + (uint64_t)(ks * 2), bd0 + (uint64_t)(ks * 2), idesc, acc);
                }
              }
            }
            if (qw == 0) QMLA_TRS(5, s);
            tc_commit(bar(b_kempty + r.idx));  // slot free once these MMAs complete
            r.next(nk);
          }
          if (ok) {
            tc_commit(bar(b_sfull + sb));
            tc_commit(bar(b_kdone + (jt % kKdoneDepth)));
          }
          if (qw == 0) QMLA_TR(5);
        }
        ++sidx;
      }
      if (jt > 0) {  // drain before TMEM is released
        const uint32_t fb = bar(b_fin + qw);
        tc_commit(fb);
        volatile int never = 0;
        mbar_wait(fb, 0, &never, nullptr, 100000000ull);
      }
    }
    __syncwarp();
  } else if (warp == kWarpPV) {
    // ====================================================== PV issuer
    if (lane == 0) {
      const uint32_t idesc = FP8 ? make_idesc_f16(0, 128, NPV, 1, 1)
                                 : make_idesc_f16(1, 128, NPV, 1, 1);
      SegCursor cur{row0, range_lo, range_hi};
      int row, k0, k1, plo, phi;
      uint32_t jt = 0, sidx = 0;
      Ring r;  // V ring position (V by TMA: token-step-major; cp.async: block-major, then token half)
      bool ok = true;
      while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
        for (int k = k0; k < k1 && ok; ++k, ++jt) {
          const uint32_t pb = jt & 1;
          ok = mbar_wait(bar(b_pfull + pb), (jt >> 1) & 1, abort_flag, status);
          QMLA_TR(7);
          if (ok && k == k0 && sidx > 0)
            ok = mbar_wait(bar(b_ofree), (sidx - 1) & 1, abort_flag, status);
          // B = P^T (K = tokens, N = heads), MN-major, no swizzle: core matrix =
          //   8 tokens x 16 bytes; LBO = token-group stride, SBO = head-block stride
          const uint64_t bd0 = make_sdesc(pbuf + pb * a.p_bytes, 16 * NPV, 128, 0);
          if (kVBoxes && a.v_tma) {
            // V slots of one token step x v_blocks blocks (TMA layout): A = block b of the slot,
            // MN-major SW128, its two 64-dim halves (bf16) 1 KB apart, 8-token groups
            // (columns per slot) KB apart; B = the step's rows of P^T.
            const int vb = a.v_blocks, nbg = NB / vb;
            const uint32_t sbo = (uint32_t)(vb * kCpb * 1024);
            for (int vs = 0; vs < kVStepsT * nbg && ok; ++vs) {
              const int ts = vs / nbg, bg = vs - ts * nbg;
              const uint32_t vidx = r.idx, vph = r.ph;
              r.next(nv);
              ok = mbar_wait(bar(b_vfull + vidx), vph, abort_flag, status);
              if (!ok) break;
              fence_proxy_async_smem();  // the row-end slot is written by cp.async
              tc_fence_after();
              const uint32_t slot = vring + vidx * a.v_slot_bytes;
              const uint64_t bd = bd0 + (uint64_t)((ts * (kVTokT / 8) * 16 * NPV) >> 4);
              const uint32_t acc = (k == k0 && ts == 0) ? 0u : 1u;
              for (int b = 0; b < vb; ++b) {
                const uint64_t ad = make_sdesc(slot + (uint32_t)(b * kCpb * 1024), 1024, sbo, 2);
                const uint32_t d_o = tmem_base + col_o + (uint32_t)((bg * vb + b) * OW);
                if constexpr (FP8) {
                  tc_mma_f8_ss(d_o, ad, bd, idesc, acc);
                  tc_mma_f8_ss(d_o, ad, bd + (uint64_t)((8 * NPV) >> 4), idesc, 1u);
                } else {
                  tc_mma_f16_ss(d_o, ad, bd, idesc, acc);
                }
              }
              tc_commit(bar(b_vempty + vidx));
            }
          } else {
            for (int bh = 0; bh < 2 * NB && ok; ++bh) {  // block bh/2, token half bh%2
              const int b = bh >> 1, hh = bh & 1;
              const uint32_t vidx = r.idx, vph = r.ph;
              r.next(nv);
              ok = mbar_wait(bar(b_vfull + vidx), vph, abort_flag, status);
              if (!ok) break;
              fence_proxy_async_smem();  // cp.async-written V slot -> tensor-core reads
              tc_fence_after();
              // A = V^T (M = 128 dims, K = tokens), MN-major, 128-byte swizzle:
              //   LBO = stride between 64-dim halves (bf16), SBO = 8-token group stride
              const uint64_t ad0 = make_sdesc(vring + vidx * kVSlotBytes, 8192, 1024, 2);
              const uint32_t d_o = tmem_base + col_o + b * OW;
#pragma unroll
              for (int ks = 0; ks < kPvSteps; ++ks) {
                const uint64_t ad = ad0 + (uint64_t)(ks * (kPvAStep >> 4));
                const uint64_t bd = bd0 + (uint64_t)((hh * kPvHalfB + ks * kPvBStep) >> 4);
                const uint32_t acc = (k == k0 && hh == 0 && ks == 0) ? 0u : 1u;
                if constexpr (FP8) {
                  // P = P_hi + P_lo: the lo half starts NPV/16 head blocks further on
                  tc_mma_f8_ss(d_o, ad, bd, idesc, acc);
                  tc_mma_f8_ss(d_o, ad, bd + (uint64_t)((8 * NPV) >> 4), idesc, 1u);
                } else {
                  tc_mma_f16_ss(d_o, ad, bd, idesc, acc);
                }
              }
              tc_commit(bar(b_vempty + vidx));
            }
          }
          if (ok) tc_commit(bar(b_odone + pb));
          QMLA_TR(8);
        }
        ++sidx;
      }
      if (jt > 0) {
        const uint32_t fb = bar(b_fin + 2);
        tc_commit(fb);
        volatile int never = 0;
        mbar_wait(fb, 0, &never, nullptr, 100000000ull);
      }
    }
    __syncwarp();
  }
  } else {
    if constexpr (NQK >= 32) setmaxnreg_inc<kRegsSoftmax>();
    // ====================================================== softmax / epilogue
    // Every wait result is folded into a barrier the whole group takes, so the
    // 256 threads always leave a tile (or the kernel) together.
    const int tid = threadIdx.x;  // 0..255
    const int sp = warp & 3;      // TMEM sub-partition
    const int hw = warp >> 2;     // head half
    const int tt = sp * 32 + lane;  // token of the tile (TMEM lane of S)
    const int H = a.H;
    const int R = a.R;     // query rows of a work row: fold drafts x H heads
    const int F = a.fold;
    constexpr int nqk = NQK;
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    // This thread's query rows: head[j] = hw * NJ + j (draft head[j] / H, head head[j] % H).
    int head[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) head[j] = hw * NJ + j;
    // head (0..H-1) of query row hw * NJ + j: the rows of a thread are consecutive, so the head
    // wraps at most NJ / H times (no division in the tile loop)
    const int hq0 = (hw * NJ) % H;
    auto head_in_row = [&](int j) -> int {
      int h = hq0 + j;
      while (h >= H) h -= H;
      return h;
    };
    // the heads of this thread's query rows are consecutive (no wrap into the next draft)
    const bool rms_contig = hq0 + min(NJ, R - hw * NJ) <= H;
    // P^T / O^T column of head half hw, position j: hw * NH + j (j >= NJ is padding)
    auto head_of_n = [&](int n) -> int {
      const int j2 = n % NH;
      if (j2 >= NJ) return -1;
      const int h = (n / NH) * NJ + j2;
      return h < R ? h : -1;
    };
    const float kscale = (FP8 && a.k_scale) ? __ldg(a.k_scale) : 1.0f;
    const bool cap = a.logit_cap > 0.f;
    float m_ref[NJ], l_part[NJ], gs[NJ];
    // Q of work row wrow -> the Q buffer (bf16 rows, or e4m3 hi / lo rows with per-row scales in
    // hv[192 + r] for FP8); query row r is head r % H of decode row wrow * F + r / H; all 256
    // softmax threads; arrives on qfull.
    // bf16 rows with 16-byte aligned q: every 16-byte unit of the stage is one cp.async, all in
    // flight at once (one round trip to memory).  Loads interleaved with the shared-memory stores,
    // as a plain loop compiles, took one round trip per unit of a thread: 12 trips, ~15 us per row
    // segment at 24 heads x 1000 columns; config 1 measured 0.571 vs 0.589 ms per call.
    auto stage_q = [&](int wrow) {
      // source of elements d0 .. of query row r (d0 a multiple of 8; rank is a multiple of 128,
      // so a 16-element unit never straddles the latent / rope boundary)
      auto q_src = [&](int r, int d0) -> const uint8_t* {
        const int dq = r / H, h = r - dq * H;
        const int64_t qrow = (int64_t)wrow * F + dq;
        return d0 < a.rank ? a.q + ((int64_t)qrow * a.q_sr + (int64_t)h * a.q_sh + d0) * 2
                           : a.q_pe + ((int64_t)qrow * a.qpe_sr + (int64_t)h * a.qpe_sh + (d0 - a.rank)) * 2;
      };
      const bool vec = a.q_vec && a.qpe_vec && a.q_dtype == 0;
      if constexpr (!FP8) {
        const int upr = a.n_sub_qk * 8;  // 16-byte units (8 elements) per head row
        if (vec) {
          // straight 16-byte copies into the swizzled rows; the bytes past qk_dim and the rows
          // past R are zero-filled
          for (int i = tid; i < nqk * upr; i += kSoftmaxThreads) {
            const int r = i / upr, u = i - r * upr, d0 = u * 8;
            const bool in = r < R && d0 < a.qk_dim;
            const uint32_t nb = in ? (uint32_t)min(16, 2 * (a.qk_dim - d0)) : 0u;
            cp_async_16(sw128(qbuf + (u >> 3) * a.q_chunk_bytes, r, u & 7), in ? q_src(r, d0) : a.q, nb);
          }
          asm volatile("cp.async.wait_all;" ::: "memory");
        } else {
          for (int i = tid; i < nqk * upr; i += kSoftmaxThreads) {
            const int r = i / upr, u = i - r * upr, d0 = u * 8;
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (r < R && d0 < a.qk_dim) {
              const uint8_t* src = q_src(r, d0);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (d0 + e < a.qk_dim) {
                  uint16_t bits = __bfloat16_as_ushort(
                      __float2bfloat16_rn(load_as_float(src + 2 * e, a.q_dtype)));
                  w[e >> 1] |= (uint32_t)bits << ((e & 1) * 16);
                }
              }
            }
            st_shared_v4(sw128(qbuf + (u >> 3) * a.q_chunk_bytes, r, u & 7), w[0], w[1], w[2], w[3]);
          }
        }
      } else {
        // The e4m3 hi / lo rows and the per-row scales were prepared for every work row by
        // q_fp8_prep_kernel (the image of this buffer): one 16-byte cp.async per unit, all in
        // flight at once.  (Converting here took one round trip to memory per unit of a thread:
        // ~30 us per row segment at 24 query rows, ~80 us at 48.)
        const uint8_t* img = a.q_img + (int64_t)wrow * a.q_img_bytes;
        for (int i = tid; i < (a.q_img_bytes >> 4); i += kSoftmaxThreads) cp_async_16(qbuf + 16 * i, img + 16 * i, 16u);
        if (tid < R) hv[192 + tid] = __ldg(a.q_scale + (int64_t)wrow * NQK + tid);
        asm volatile("cp.async.wait_all;" ::: "memory");
      }
      fence_proxy_async_smem();
      named_bar_sync(kBarSoftmax, kSoftmaxThreads);
      if (lane == 0) mbar_arrive(bar(b_qfull));
    };
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, sidx = 0;
    bool ok = true;
    // Q of the first segment; a later segment's Q is staged either before or after the
    // previous segment's epilogue (see below).
    bool have = next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi);
    if (have) stage_q(row);
    while (ok && have) {
      const int L = work_len(a.seq_lens, F, row);
      // tokens query row head[j] sees: the length of its own decode row (MTP drafts are causal:
      // draft d of a request sees L - (fold-1-d) tokens); 0 for padding rows
      int lim[NJ];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        m_ref[j] = -INFINITY;
        l_part[j] = 0.f;
        float g = a.sm_scale;
        if constexpr (FP8) g *= kscale / (head[j] < R ? hv[192 + head[j]] : 1.f);
        gs[j] = g;
        lim[j] = 0;
        if (head[j] < R) {
          const int Ld = F == 1 ? L : __ldg(a.seq_lens + (int64_t)row * F + head[j] / H);
          lim[j] = Ld < 0 ? 0 : Ld;
        }
      }

      // ---------------- tiles
      for (int k = k0; k < k1; ++k, ++jt) {
        const uint32_t sb = jt % SB;  // S buffer
        const uint32_t pb = jt & 1;   // P buffer / odone / rms parity
        const int nvalid = min(kTile, L - k * kTile);
        const bool valid = tt < nvalid;
        float x[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) x[j] = 0.f;
        ok = mbar_wait(bar(b_sfull + sb), (jt / SB) & 1, abort_flag, status);
        if (tid == a.trace_tid) QMLA_TR(9);
        if (ok) {
          tc_fence_after();
          const uint32_t tb = tmem_base + lane_base + col_s + sb * SW + hw * NJ;
          // S = sum of the KP partials (and of the hi / lo halves for FP8)
          // (one partial's columns in flight at a time: FP8's hi + lo of 24 rows are 48 registers)
#pragma unroll
          for (int p = 0; p < KP; ++p) {
            float xp[FP8 ? 2 : 1][NJ];
            load_cols<NJ>(tb + p * SWP, xp[0]);
            if constexpr (FP8) load_cols<NJ>(tb + p * SWP + nqk, xp[1]);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
              float v = xp[0][j];
              if constexpr (FP8) v += xp[1][j];
              x[j] = p == 0 ? v : x[j] + v;
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(b_sempty + sb));
        }
        if (tid == a.trace_tid) QMLA_TR(14);
        // ---- rms divisor -> per-(token, head) factor
        float f[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) f[j] = gs[j];
        if (a.rms_units > 0 && ok) {
          ok = mbar_wait(bar(b_rfull + pb), (jt >> 1) & 1, abort_flag, status);
          if (tid == a.trace_tid && a.use_tma) QMLA_TR(1);  // (event 1 is the cp.async K loader's otherwise)
          if (ok) {
            if (valid) {
              // this token's staged rms tail (shared memory): one value per head, shared by a
              // work row's drafts; es bytes per head (bf16 values / raw bf16 bytes, or one code)
              const uint32_t rrow = rmsbuf + pb * (kTile * rstride) + tt * rstride + a.rms_skip;
              const int es = (!FP8 || a.rms_mode == 2) ? 2 : 1;
              auto factor = [&](int j, uint32_t bits) -> float {
                if (FP8 && a.rms_mode == 3)  // 1 / rms = 2^(3 - code * 6/255)
                  return gs[j] * ex2_approx(3.0f - (float)bits * (6.0f / 255.0f));
                const float rv = (!FP8 || a.rms_mode == 2)
                                     ? __bfloat162float(__ushort_as_bfloat16((uint16_t)bits))
                                     : e4m3_to_f32((uint8_t)bits) * kscale;
                return rv > 0.f ? __fdividef(gs[j], rv) : gs[j];
              };
              if (rms_contig) {
                // heads hq0 .. hq0 + NJ - 1 lie side by side in the row: a few aligned 32-bit
                // loads realigned by funnel shifts, instead of a byte load per head
                constexpr int NW = NJ / 2 + 2;  // covers NJ two-byte heads plus the misalignment
                const uint32_t addr = rrow + (uint32_t)(hq0 * es);
                const uint32_t a4 = addr & ~3u, sh = (addr & 3u) * 8u;
                const int nw = (int)(((addr & 3u) + (uint32_t)(NJ * es) + 3u) >> 2);
                uint32_t w[NW];
#pragma unroll
                for (int k = 0; k < NW; ++k) w[k] = k < nw ? ld_shared_u32(a4 + 4 * k) : 0u;
#pragma unroll
                for (int k = 0; k + 1 < NW; ++k) w[k] = __funnelshift_r(w[k], w[k + 1], sh);
                if (es == 1) {
#pragma unroll
                  for (int j = 0; j < NJ; ++j)
                    if (head[j] < R) f[j] = factor(j, (w[j >> 2] >> ((j & 3) * 8)) & 0xffu);
                } else {
#pragma unroll
                  for (int j = 0; j < NJ; ++j)
                    if (head[j] < R) f[j] = factor(j, (w[j >> 1] >> ((j & 1) * 16)) & 0xffffu);
                }
              } else {
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                  if (head[j] < R) {
                    const uint32_t b = rrow + (uint32_t)(head_in_row(j) * es);
                    f[j] = factor(j, es == 1 ? ld_shared_u8(b) : ld_shared_u8(b) | (ld_shared_u8(b + 1) << 8));
                  }
                }
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(b_rempty + pb));
          }
        }
        if (tid == a.trace_tid) QMLA_TR(15);
        if (tid == a.trace_tid) QMLA_TR(10);
        // ---- logits (log2 units) and the lazy-rescale test
        bool need = false;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          float v = -INFINITY;
          if (k * kTile + tt < lim[j]) {  // inside this query row's causal limit (0 for padding)
            float s = x[j] * f[j];
            if (cap) s = a.logit_cap * tanhf(s / a.logit_cap);
            v = s * kLog2e;
          }
          x[j] = v;
          need |= v > m_ref[j] + kRescaleThreshold;
        }
        // PV(jt-2) must be done before P buffer pb is rewritten
        if (jt >= 2 && ok) {
          const uint32_t jp = jt - 2;
          ok = mbar_wait(bar(b_odone + (jp & 1)), (jp >> 1) & 1, abort_flag, status);
        }
        // One group barrier per tile: it reduces the rescale test and, folded into it, any failed
        // wait; only when it fires does a second reduction decide uniformly whether to abort.
        need = named_bar_or(kBarSoftmax, kSoftmaxThreads, need || !ok);
        if (tid == a.trace_tid) QMLA_TR(11);
        if (need && named_bar_or(kBarSoftmax, kSoftmaxThreads, !ok)) {
          ok = false;
          break;
        }
        if (need) {
          // exact tile max per head: over this warp's 32 tokens, then the 4 sub-partitions
          float wm[NJ];
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            float v = x[j];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
            wm[j] = v;
          }
          if (lane == 0) {
#pragma unroll
            for (int j = 0; j < NJ; ++j) red[(hw * 4 + sp) * 32 + j] = wm[j];
          }
          named_bar_sync(kBarSoftmax, kSoftmaxThreads);
          bool any_scale = false;
          float alpha[NJ];
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            float t = fmaxf(fmaxf(red[(hw * 4 + 0) * 32 + j], red[(hw * 4 + 1) * 32 + j]),
                            fmaxf(red[(hw * 4 + 2) * 32 + j], red[(hw * 4 + 3) * 32 + j]));
            float mn = fmaxf(m_ref[j], t);
            float al = (mn == -INFINITY) ? 1.f
                                         : (m_ref[j] == -INFINITY ? 0.f : exp2f(m_ref[j] - mn));
            alpha[j] = al;
            any_scale |= (al != 1.f) && (k > k0);
            m_ref[j] = mn;
            l_part[j] *= al;
          }
          any_scale = named_bar_or(kBarSoftmax, kSoftmaxThreads, any_scale);  // red[] free again
          if (any_scale) {
            // O holds tiles k0..k-1: wait for PV(k-1), then rescale it in TMEM
            if (sp == 0 && lane == 0) {
#pragma unroll
              for (int j = 0; j < NJ; ++j) hv[head[j]] = alpha[j];
            }
            named_bar_sync(kBarSoftmax, kSoftmaxThreads);
            const uint32_t jp = jt - 1;
            ok = mbar_wait(bar(b_odone + (jp & 1)), (jp >> 1) & 1, abort_flag, status);
            if (ok) {
              tc_fence_after();
              float an[NPV / 2];
#pragma unroll
              for (int i = 0; i < NPV / 2; ++i) {
                int h = head_of_n(hw * (NPV / 2) + i);
                an[i] = h >= 0 ? hv[h] : 1.f;
              }
              for (int blk = 0; blk < NB; ++blk) {
                const uint32_t ta = tmem_base + lane_base + col_o + blk * OW + hw * (NPV / 2);
#pragma unroll
                for (int g8 = 0; g8 < NPV / 16; ++g8) {
                  float ov[8];
                  tmem_ld8(ta + g8 * 8, ov);
                  tmem_wait_ld();
#pragma unroll
                  for (int e = 0; e < 8; ++e) ov[e] *= an[g8 * 8 + e];
                  tmem_st8(ta + g8 * 8, ov);
                }
              }
              tmem_wait_st();
            }
            if (named_bar_or(kBarSoftmax, kSoftmaxThreads, !ok)) {  // hv[] free again
              ok = false;
              break;
            }
          }
        }
        // ---- P = 2^(x - m) -> P^T buffer pb
        {
          float p[NH];
#pragma unroll
          for (int j = 0; j < NH; ++j) {
            if (j < NJ) {
              p[j] = (x[j] == -INFINITY) ? 0.f : ex2_approx(x[j] - m_ref[j]);
              l_part[j] += p[j];
            } else {
              p[j] = 0.f;  // padding columns of P^T
            }
          }
          const uint32_t prow = pbuf + pb * a.p_bytes + (tt >> 3) * (16 * NPV) + (tt & 7) * 16;
          const int n0 = hw * NH;  // first P^T column of this head half (multiple of 8)
          if constexpr (!FP8) {
            // 8 heads (16 bytes) per core-matrix row; NH/8 core matrices 128 bytes apart
            uint32_t w[NH / 2];
#pragma unroll
            for (int j = 0; j < NH; j += 2)
              w[j / 2] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p[j])) |
                         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p[j + 1])) << 16);
#pragma unroll
            for (int c = 0; c < NH / 8; ++c)
              st_shared_v4(prow + ((n0 >> 3) + c) * 128, w[4 * c], w[4 * c + 1], w[4 * c + 2],
                           w[4 * c + 3]);
          } else {
            // 16 heads (16 bytes) per core-matrix row; hi columns [0, NPV), lo [NPV, 2 NPV)
            // two elements per conversion (e4m3x2): the same round-to-nearest bytes as one at a time
            uint32_t whi[NH / 4], wlo[NH / 4];
#pragma unroll
            for (int q4 = 0; q4 < NH / 4; ++q4) {
              whi[q4] = 0u;
              wlo[q4] = 0u;
#pragma unroll
              for (int e = 0; e < 4; e += 2) {
                const float2 v = make_float2(p[q4 * 4 + e], p[q4 * 4 + e + 1]);
                const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
                const float2 hv2 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(hi, __NV_E4M3)));
                const __nv_fp8x2_storage_t lo =
                    __nv_cvt_float2_to_fp8x2(make_float2(v.x - hv2.x, v.y - hv2.y), __NV_SATFINITE, __NV_E4M3);
                whi[q4] |= (uint32_t)hi << (8 * e);
                wlo[q4] |= (uint32_t)lo << (8 * e);
              }
            }
            if constexpr (NH == 16) {
              st_shared_v4(prow + (n0 >> 4) * 128, whi[0], whi[1], whi[2], whi[3]);
              st_shared_v4(prow + ((NPV + n0) >> 4) * 128, wlo[0], wlo[1], wlo[2], wlo[3]);
            } else {
              // 8 columns (8 bytes) at a time: column n sits in core matrix n / 16 at byte n % 16
#pragma unroll
              for (int g8 = 0; g8 < NH / 8; ++g8) {
                const int n = n0 + 8 * g8, nl = NPV + n;
                st_shared_v2(prow + (n >> 4) * 128 + (n & 15), whi[2 * g8], whi[2 * g8 + 1]);
                st_shared_v2(prow + (nl >> 4) * 128 + (nl & 15), wlo[2 * g8], wlo[2 * g8 + 1]);
              }
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (tid == a.trace_tid) QMLA_TR(12);
        if (lane == 0) mbar_arrive(bar(b_pfull + pb));
      }
      if (!ok) break;

      // ---------------- the next segment's Q, early after a short segment (its QK is
      // complete): the next QK then overlaps this segment's PV tail and epilogue.  After a
      // long segment the boundary costs little, and staging Q while the V loads stream
      // measured 2% slower on config 1, so Q is staged after the epilogue there.
      const bool early = k1 - k0 <= a.early_q;
      if (early) {
        const int nrow = peek_segment_row(a.tile_prefix, cur);
        if (nrow >= 0) stage_q(nrow);
      }

      // ---------------- epilogue: O^T / l -> output (or partial)
      {
        const uint32_t jl = jt - 1;
        ok = mbar_wait(bar(b_odone + (jl & 1)), (jl >> 1) & 1, abort_flag, status);
        float ls[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          float v = l_part[j];
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          ls[j] = v;
        }
        if (lane == 0) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) red[(hw * 4 + sp) * 32 + j] = ls[j];
        }
        if (named_bar_or(kBarSoftmax, kSoftmaxThreads, !ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (sp == 0 && lane == 0) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            if (head[j] < R) {
              float lt = red[(hw * 4 + 0) * 32 + j] + red[(hw * 4 + 1) * 32 + j] +
                         red[(hw * 4 + 2) * 32 + j] + red[(hw * 4 + 3) * 32 + j];
              hv[64 + head[j]] = lt;
              hv[128 + head[j]] = m_ref[j];
            }
          }
        }
        named_bar_sync(kBarSoftmax, kSoftmaxThreads);
        const bool full = (plo >= range_lo) && (phi <= range_hi);
        const int slot = (plo <= range_lo) ? 2 * (int)blockIdx.x : 2 * (int)blockIdx.x + 1;
        const float oscale = FP8 ? kscale : 1.0f;
        float linv[NPV / 2];
        int hn[NPV / 2];
#pragma unroll
        for (int i = 0; i < NPV / 2; ++i) {
          hn[i] = head_of_n(hw * (NPV / 2) + i);
          float lt = hn[i] >= 0 ? hv[64 + hn[i]] : 0.f;
          linv[i] = lt > 0.f ? oscale / lt : 0.f;
        }
        for (int blk = 0; blk < NB; ++blk) {
          const int d = blk * 128 + sp * 32 + lane;
          const uint32_t ta = tmem_base + lane_base + col_o + blk * OW + hw * (NPV / 2);
          float ov[NPV / 2];
          if constexpr (NPV == 48) {
            tmem_ld16(ta, ov);
            tmem_ld8(ta + 16, ov + 16);
          } else if constexpr (NPV == 32) {
            tmem_ld16(ta, ov);
          } else {
            tmem_ld8(ta, ov);
          }
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < NPV / 2; ++i) {
            const int r = hn[i];  // query row: head r % H of decode row row * F + r / H
            if (r >= 0) {
              const float v = ov[i] * linv[i];
              if (full) {
                const int dq = r / H;
                store_from_float(a.o + (((int64_t)row * F + dq) * a.o_sr + (int64_t)(r - dq * H) * a.o_sh + d) *
                                           dt_size(a.o_dtype),
                                 a.o_dtype, v);
              } else {
                a.part_o[((int64_t)slot * R + r) * a.rank + d] = v;
              }
            }
          }
        }
        if (tid < R) {
          const float lt = hv[64 + tid];
          const float l2 = hv[128 + tid] + log2f(lt);  // log2-domain LSE
          if (full) {
            const int dq = tid / H;
            if (a.lse)
              store_from_float(a.lse + (((int64_t)row * F + dq) * a.lse_sr + (tid - dq * H)) *
                                           dt_size(a.lse_dtype),
                               a.lse_dtype, l2 * kLn2);
          } else {
            a.part_lse[(int64_t)slot * R + tid] = l2;
          }
        }
        tc_fence_before();
        named_bar_sync(kBarSoftmax, kSoftmaxThreads);  // hv[] reads done; O reads done
        if (lane == 0) mbar_arrive(bar(b_ofree));
        // ---------------- a row cut at CTA range boundaries, in-kernel merge mode: the CTA that
        // writes the row's last piece merges all pieces, in CTA order (the reference's stage 2,
        // mla_decode_attention.py:1064-1137), so the result does not depend on which CTA is last
        if (!full && a.row_done) {
          __threadfence();  // this CTA's piece is visible before it is counted
          named_bar_sync(kBarSoftmax, kSoftmaxThreads);
          auto cta_of = [&](int t) {  // the non-empty range holding tile t
            int lo = 0, hi = a.G;
            while (hi - lo > 1) {
              const int m = (lo + hi) >> 1;
              if (__ldg(a.range_bounds + m) <= t) lo = m; else hi = m;
            }
            return lo;
          };
          const int c0 = cta_of(plo), c1 = cta_of(phi - 1);
          if (tid == 0) {
            int np = 0;
            for (int c = c0; c <= c1; ++c) np += __ldg(a.range_bounds + c) < __ldg(a.range_bounds + c + 1);
            const bool last = atomicAdd(a.row_done + row, 1) == np - 1;
            if (last) __threadfence();  // the other pieces are visible before they are read
            *fix_flag = last ? 1 : 0;
          }
          named_bar_sync(kBarSoftmax, kSoftmaxThreads);
          if (*fix_flag) {
            const int n4 = a.rank / 4, osz = dt_size(a.o_dtype);
            for (int idx = tid; idx < R * n4; idx += kSoftmaxThreads) {
              const int r = idx / n4, d = 4 * (idx - r * n4);
              float m = -INFINITY;
              for (int c = c0; c <= c1; ++c) {
                const int b0 = __ldg(a.range_bounds + c);
                if (b0 >= __ldg(a.range_bounds + c + 1)) continue;  // an empty range wrote nothing
                const int sl = plo <= b0 ? 2 * c : 2 * c + 1;
                m = fmaxf(m, __ldcg(a.part_lse + (int64_t)sl * R + r));
              }
              float sum = 0.f;
              float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
              for (int c = c0; c <= c1; ++c) {
                const int b0 = __ldg(a.range_bounds + c);
                if (b0 >= __ldg(a.range_bounds + c + 1)) continue;
                const int sl = plo <= b0 ? 2 * c : 2 * c + 1;
                const float w = m == -INFINITY ? 0.f : exp2f(__ldcg(a.part_lse + (int64_t)sl * R + r) - m);
                const float4 v = __ldcg(reinterpret_cast<const float4*>(a.part_o + ((int64_t)sl * R + r) * a.rank + d));
                sum += w;
                acc.x += w * v.x;
                acc.y += w * v.y;
                acc.z += w * v.z;
                acc.w += w * v.w;
              }
              const float inv = sum > 0.f ? 1.f / sum : 0.f;
              const int dq = r / H;
              uint8_t* orow = a.o + (((int64_t)row * F + dq) * a.o_sr + (int64_t)(r - dq * H) * a.o_sh + d) * osz;
              store_from_float(orow, a.o_dtype, acc.x * inv);
              store_from_float(orow + osz, a.o_dtype, acc.y * inv);
              store_from_float(orow + 2 * osz, a.o_dtype, acc.z * inv);
              store_from_float(orow + 3 * osz, a.o_dtype, acc.w * inv);
              if (d == 0 && a.lse)
                store_from_float(a.lse + (((int64_t)row * F + dq) * a.lse_sr + (r - dq * H)) * dt_size(a.lse_dtype),
                                 a.lse_dtype, (m + log2f(sum)) * kLn2);
            }
          }
        }
      }
      ++sidx;
      have = next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi);
      if (have && !early) stage_q(row);
    }
  }
  // ------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
#ifdef QMLA_TRACE
  if (a.trace && threadIdx.x == 0) a.trace[6 * 4096 + blockIdx.x * 2 + 1] = globaltimer_ns();
#endif
  if (warp == kWarpQK) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace qmla
