// Paged latent-KV MLA decode for B200 (sm_100a).
//
// One persistent CTA per SM walks a balanced, contiguous range of 64-token
// tiles over all decode rows (rows are cut into segments at CTA boundaries and
// merged afterwards).  Warp roles:
//   warps 0-7   softmax / epilogue.  Warp w reads TMEM sub-partition w%4 and
//               owns half of the heads (w/4); all 32 lanes are busy (two lanes
//               per token, alternate heads, via the 16x64b TMEM load shape)
//   warp  8     TMA producer: page-table lookups + 3-D tiled bulk loads
//   warp  9     QK issuer (tcgen05) + TMEM owner
//   warp  10    PV issuer (tcgen05)
//   warp  11    (FP8 cache) rms-tail fix-up: copies the per-head rms bytes out
//               of the tile and zeroes the bytes between the attention width
//               and the MMA K boundary, so log8 codes never reach the MMA
// Per 64-token tile:
//   S^T[64 tok, heads] = K_tile . Q^T      tcgen05 M=64, K-major A and B
//   softmax over tokens with the per-(token, head) rms divisor, base 2, lazy
//   rescale (O is only rescaled when a running max grows by more than 2^8)
//   O^T[rank, heads]  += V^T . P^T         tcgen05 M=128, MN-major A and B
// bf16 caches use kind::f16 (bf16 operands).  FP8 caches use kind::f8f6f4 on
// the raw e4m3 tile; q and P are each split into two e4m3 terms (hi + lo)
// stacked along N, so the contraction keeps ~bf16 precision without any
// dequantisation pass over the cache.  The latent part of a tile stays in
// shared memory from QK to PV, so each cache byte crosses HBM once.
// Semantics follow the reference Triton kernel
// qwen_mla/ops/mla_decode_attention.py:297-586 and its split merge :1064-1137.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "qmla_ptx.cuh"

namespace qmla {

constexpr int kTile = 64;          // tokens per tile
constexpr int kMaxQkChunks = 16;   // QK width <= 1024 elements
constexpr int kMaxCtas = 160;      // persistent CTAs per launch (B200: 148 SMs)
constexpr int kSoftmaxWarps = 8;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kWarpProducer = 8, kWarpQK = 9, kWarpPV = 10, kWarpFix = 11;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P may reach 2^8 before O is rescaled
constexpr int kBarSoftmax = 1;             // named barrier id of the softmax warps

struct DecodeArgs {
  // query
  const uint8_t* q;
  const uint8_t* q_pe;
  int64_t q_sr, q_sh, qpe_sr, qpe_sh;  // element strides
  int q_dtype;
  int q_vec, qpe_vec;  // 16-byte vector loads are legal for q / q_pe rows
  // cache / paging
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* seq_lens;
  int page_size;
  int run_rows;  // gcd(page_size, 64): tokens per TMA box
  // geometry
  int num_rows, H, rank, qk_dim, rms_offset, rms_mode, rms_bytes;
  int nqk;          // heads rounded up to a multiple of 8
  int n_slot_tile;  // 128-dim slots loaded per tile (covers qk and the rms tail)
  int n_qk_slots;   // slots the QK contraction reads
  int n_sub_qk;     // 128-byte-wide MMA sub-chunks of the QK width
  int fix_slot0;    // FP8: first slot the fix-up reads (-1: none)
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
  const int32_t* tile_prefix;  // [num_rows + 1]
  float* part_o;               // [2*G][H][rank]
  float* part_lse;             // [2*G][H] (log2 units)
  int G;
  // shared-memory layout (byte offsets from the 1024-aligned base)
  uint32_t off_ring, nslot, off_q, q_chunk_bytes, off_p, p_bytes, off_rms, off_misc;
  // Optional stage timestamps of CTA 0 (builds with -DQMLA_TRACE only):
  // trace[tile * 16 + event] = %globaltimer in ns.
  unsigned long long* trace;
};

#ifdef QMLA_TRACE
#define QMLA_TR(ev)                                                                 \
  do {                                                                               \
    if (a.trace && blockIdx.x == 0 && jt < 256) a.trace[jt * 16 + (ev)] = globaltimer_ns(); \
  } while (0)
#else
#define QMLA_TR(ev) \
  do {              \
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
__device__ __forceinline__ void st_shared_u32(uint32_t a, uint32_t x) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(x) : "memory");
}

// Load N (2, 4, 6 or 8) 16x64b column pairs of one S block into v[0..N).
template <int N>
__device__ __forceinline__ void load_s_pairs(uint32_t taddr, float* v) {
  if constexpr (N == 8) {
    tmem_ld16x64<8>(taddr, v);
  } else if constexpr (N == 6) {
    tmem_ld16x64<4>(taddr, v);
    tmem_ld16x64<2>(taddr + 8, v + 4);
  } else if constexpr (N == 4) {
    tmem_ld16x64<4>(taddr, v);
  } else {
    tmem_ld16x64<2>(taddr, v);
  }
}

// ---------------------------------------------------------------- the kernel
template <bool FP8, int NB, int NQK>
__global__ void __launch_bounds__(FP8 ? 384 : 352, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeArgs a) {
  static_assert(NQK % 8 == 0 && NQK >= 8 && NQK <= 32, "heads rounded to 8..32");
  constexpr int NPV = NQK <= 16 ? 16 : 32;  // PV MMA N (multiple of 16)
  constexpr int kSlotBytes = FP8 ? 8192 : 16384;  // 64 tokens x 128 dims
  constexpr int kSubs = FP8 ? 1 : 2;              // 128-byte-wide sub-chunks per slot
  constexpr int OW = FP8 ? 2 * NPV : NPV;         // TMEM columns per O block (hi|lo for FP8)
  constexpr int SWP = FP8 ? 2 * NPV : NPV;        // TMEM columns per S partial (hi|lo for FP8)
  // Consecutive MMAs into one accumulator serialise (~64 cycles each); independent
  // accumulators pipeline down to the operand-fetch bound.  So the QK reduction is
  // split over KP partial accumulators (summed by the softmax) and S is double
  // buffered (SB) when TMEM allows.
  constexpr int kFree = 512 - NB * OW;
  constexpr int KP = (kFree >= 8 * SWP) ? 4 : (kFree >= 4 * SWP) ? 2 : (kFree >= 2 * SWP) ? 2 : 1;
  constexpr int SB = (kFree >= 2 * KP * SWP) ? 2 : 1;
  constexpr int SW = KP * SWP;                     // TMEM columns per S buffer
  constexpr uint32_t kCols = NB * OW + SB * SW;
  constexpr uint32_t kTmemCols = kCols <= 32 ? 32 : kCols <= 64 ? 64 : kCols <= 128 ? 128
                                 : kCols <= 256 ? 256 : 512;
  static_assert(kCols <= 512, "TMEM budget");
  constexpr int NJ = NQK / 4;   // heads per softmax thread
  constexpr int NJP = NPV / 4;  // P^T columns per softmax thread (NJ real + zero padding)
  constexpr int kKStepBytes = 32;
  constexpr int kPvSteps = FP8 ? 2 : 4;      // K = 32 (e4m3) or 16 (bf16) tokens per PV MMA
  constexpr int kPvAStep = FP8 ? 4096 : 2048;
  constexpr int kPvBStep = (FP8 ? 4 : 2) * 16 * NPV;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ------------------------------------------------ work range
  const int total = __ldg(a.tile_prefix + a.num_rows);
  const int tpc = (total + a.G - 1) / a.G;
  const int range_lo = blockIdx.x * tpc;
  const int range_hi = min(total, range_lo + tpc);
  if (range_lo >= range_hi) return;  // uniform for the whole CTA
  const int row0 = first_row_at(a.tile_prefix, a.num_rows, range_lo);

  // ------------------------------------------------ barriers and scratch
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_misc);
  const uint32_t nslot = a.nslot;
  const uint32_t b_full = 0;                // [nslot] TMA landed
  const uint32_t b_empty = nslot;           // [nslot] slot free
  const uint32_t b_sfull = 2 * nslot;       // [2] S ready
  const uint32_t b_sempty = b_sfull + 2;    // [2] S consumed
  const uint32_t b_pfull = b_sempty + 2;    // [2] P written (+ O rescaled)
  const uint32_t b_odone = b_pfull + 2;     // [2] PV finished
  const uint32_t b_qfull = b_odone + 2;     // [1] Q staged
  const uint32_t b_ofree = b_qfull + 1;     // [1] O read by the epilogue
  const uint32_t b_fix = b_ofree + 1;       // [2] FP8 fix-up done (rms staged)
  const uint32_t b_rempty = b_fix + 2;      // [2] FP8 rms staging consumed
  const uint32_t b_fin = b_rempty + 2;      // [2] issuer drain at teardown
  const uint32_t b_rdone = b_fin + 2;       // [2] bf16: rms tail of the tile read
  const uint32_t n_bars = b_rdone + 2;
  auto bar = [&](uint32_t i) -> uint32_t { return smem_u32(bars + i); };
  uint8_t* misc2 = smem + a.off_misc + ((n_bars * 8 + 15) / 16) * 16;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc2 + 4);
  float* red = reinterpret_cast<float*>(misc2 + 16);   // [2 halves][4 sp][32]
  float* hv = red + 256;                               // [4][32] per-head broadcast values
  // hv[0..31] alpha, hv[32..63] l, hv[64..95] m, hv[96..127] q scale (FP8)

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nslot; ++i) {
      mbar_init(bar(b_full + i), 1);
      mbar_init(bar(b_empty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(b_sfull + i), 1);
      mbar_init(bar(b_sempty + i), kSoftmaxWarps);
      mbar_init(bar(b_pfull + i), kSoftmaxWarps);
      mbar_init(bar(b_odone + i), 1);
      mbar_init(bar(b_fix + i), 1);
      mbar_init(bar(b_rempty + i), kSoftmaxWarps);
      mbar_init(bar(b_fin + i), 1);
      mbar_init(bar(b_rdone + i), kSoftmaxWarps);
    }
    mbar_init(bar(b_qfull), kSoftmaxWarps);
    mbar_init(bar(b_ofree), kSoftmaxWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpQK) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (warp == kWarpProducer && lane == 0) prefetch_tmap(&tmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t col_o = 0;
  const uint32_t col_s = NB * OW;

  const uint32_t ring = sbase + a.off_ring;
  const uint32_t qbuf = sbase + a.off_q;
  const uint32_t pbuf = sbase + a.off_p;
  int* status = a.status;
  auto slot_addr = [&](uint32_t it) -> uint32_t { return ring + (it % nslot) * kSlotBytes; };
  // Tile-local load order: the rope / rms slots (dims slots >= NB) first, then the
  // latent slots.  Rope slots are released as soon as S (and the rms tail) are
  // consumed, so the next tile's first loads can start while this tile's latent
  // part is still held for PV.
  const int nrope = a.n_slot_tile - NB;
  auto pos_of = [&](int s) -> int { return s >= NB ? s - NB : nrope + s; };
  auto dims_of = [&](int t) -> int { return t < nrope ? NB + t : t - nrope; };
  // shared address of tile-local position t given the tile's first ring index
  auto slot_at = [&](uint32_t tbase, int t) -> uint32_t {
    uint32_t idx = tbase + (uint32_t)t;
    if (idx >= nslot) idx -= nslot;
    return ring + idx * kSlotBytes;
  };

  if (warp == kWarpProducer) {
    // ====================================================== TMA producer
    const uint64_t pol = policy_evict_first();
    const int runs = kTile / a.run_rows;  // 1, 2 or 4
    const int xstep = FP8 ? 128 : 64;     // box width in elements
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, armed = 0, ridx = 0, rph = 0;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      int L = __ldg(a.seq_lens + row);
      L = L < 0 ? 0 : L;
      const int32_t* bt = a.block_table + (int64_t)row * a.bt_stride;
      auto page_of = [&](int k, int& y) -> int {
        int tok0 = k * kTile + lane * a.run_rows;
        y = 0;
        if (lane < runs && tok0 < L) {
          y = tok0 % a.page_size;
          return __ldg(bt + tok0 / a.page_size);
        }
        return -1;  // out of the tensor: TMA fills zeros
      };
      int ny, npage = page_of(k0, ny);
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        int cpage = npage, cy = ny;
        if (k + 1 < k1) npage = page_of(k + 1, ny);  // prefetch next tile's pages
        int pages[4], ys[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          pages[r] = __shfl_sync(0xffffffffu, cpage, r);
          ys[r] = __shfl_sync(0xffffffffu, cy, r);
        }
        for (int t = 0; t < a.n_slot_tile && ok; ++t) {
          const int s = dims_of(t);
          if (lane == 0) {
            ok = mbar_wait(bar(b_empty + ridx), rph ^ 1, abort_flag, status);
            if (t == 0) QMLA_TR(0);
            if (ok) {
              const uint32_t fb = bar(b_full + ridx);
              mbar_expect_tx(fb, (uint32_t)kSlotBytes);
              const uint32_t dst0 = ring + ridx * kSlotBytes;
#pragma unroll
              for (int sc = 0; sc < kSubs; ++sc)
                for (int r = 0; r < runs; ++r)
                  tma_load_3d(dst0 + sc * 8192 + r * a.run_rows * 128, &tmap, (kSubs * s + sc) * xstep,
                              ys[r], pages[r], fb, pol);
              armed = jt * a.n_slot_tile + t + 1;
              if (t == a.n_slot_tile - 1) QMLA_TR(1);
              if (t == 0) QMLA_TR(13);
            }
          }
          if (++ridx == nslot) {
            ridx = 0;
            rph ^= 1;
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
        }
      }
    }
    // After an abort: wait (bounded) for the loads already issued so no bulk
    // copy still targets this CTA's shared memory when it exits.
    if (!ok && lane == 0) {
      uint32_t first = armed > nslot ? armed - nslot : 0u;
      for (uint32_t it = first; it < armed; ++it) {
        volatile int never = 0;
        mbar_wait(bar(b_full + it % nslot), (it / nslot) & 1, &never, nullptr, 20000000ull);
      }
    }
  } else if (warp == kWarpQK) {
    // ====================================================== QK issuer
    const uint32_t idesc = FP8 ? make_idesc_f16(0, 64, 2 * NQK, 0, 0)
                               : make_idesc_f16(1, 64, NQK, 0, 0);
    const uint32_t qc16 = a.q_chunk_bytes >> 4;               // Q chunk stride, descriptor units
    const uint64_t q_desc0 = make_sdesc(qbuf, 16, 1024, 2);   // Q chunk 0 (K-major, 128B swizzle)
    const int fix_slot = (FP8 && a.fix_slot0 >= 0) ? a.fix_slot0 : 1 << 30;
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, sidx = 0, ridx = 0, rph = 0;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      if (lane == 0) ok = mbar_wait(bar(b_qfull), sidx & 1, abort_flag, status);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const uint32_t sb = jt % SB;
        const uint32_t pb = jt & 1;
        if (lane == 0) {
          if (jt >= SB) ok = mbar_wait(bar(b_sempty + sb), ((jt - SB) / SB) & 1, abort_flag, status);
          QMLA_TR(2);
          tc_fence_after();
          const uint32_t d_s = tmem_base + col_s + sb * SW;
          bool first = true;  // first sub-chunk of the tile initialises the KP partials
          for (int t = 0; t < a.n_slot_tile; ++t) {
            const int s = dims_of(t);
            const uint32_t cidx = ridx, cph = rph;
            if (++ridx == nslot) {
              ridx = 0;
              rph ^= 1;
            }
            if (!ok || s >= a.n_qk_slots) continue;  // rms-only slot (ring position still advances)
            if (s == fix_slot) ok = mbar_wait(bar(b_fix + pb), (jt >> 1) & 1, abort_flag, status);
            if (ok) ok = mbar_wait(bar(b_full + cidx), cph, abort_flag, status);
            if (!ok) continue;
            if (t == 0) QMLA_TR(3);
            if (t == a.n_slot_tile - 1) QMLA_TR(4);
            tc_fence_after();
            const uint64_t ad0 = make_sdesc(ring + cidx * kSlotBytes, 16, 1024, 2);
            const uint64_t bd0 = q_desc0 + (uint64_t)(s * kSubs) * qc16;
#pragma unroll
            for (int sc = 0; sc < kSubs; ++sc) {
              if (s * kSubs + sc < a.n_sub_qk) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                  const uint64_t ad = ad0 + (uint64_t)(sc * 512 + ks * 2);
                  const uint64_t bd = bd0 + (uint64_t)(sc * qc16 + ks * 2);
                  const uint32_t d = d_s + (ks % KP) * SWP;
                  const uint32_t acc = (first && ks < KP) ? 0u : 1u;
                  if constexpr (FP8)
                    tc_mma_f8_ss(d, ad, bd, idesc, acc);
                  else
                    tc_mma_f16_ss(d, ad, bd, idesc, acc);
                }
                first = false;
              }
            }
            // FP8: the rope slot is free once these MMAs finish (rms was staged by the fix-up)
            if (FP8 && s >= NB) tc_commit(bar(b_empty + cidx));
          }
          if (ok) tc_commit(bar(b_sfull + sb));
          QMLA_TR(5);
        } else {
          for (int t = 0; t < a.n_slot_tile; ++t)
            if (++ridx == nslot) {
              ridx = 0;
              rph ^= 1;
            }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      ++sidx;
    }
    if (lane == 0 && jt > 0) {  // drain before TMEM is released
      tc_commit(bar(b_fin));
      volatile int never = 0;
      mbar_wait(bar(b_fin), 0, &never, nullptr, 100000000ull);
    }
  } else if (warp == kWarpPV) {
    // ====================================================== PV issuer
    const uint32_t idesc = FP8 ? make_idesc_f16(0, 128, 2 * NPV, 1, 1)
                               : make_idesc_f16(1, 128, NPV, 1, 1);
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, sidx = 0, tbase = 0;  // tbase: ring index of the tile's first slot
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const uint32_t pb = jt & 1;  // P buffer / odone / rdone parity
        if (lane == 0) {
          if constexpr (!FP8) {
            // bf16: rope slots (which hold the rms tail) are free once the softmax
            // has read S and the rms values of this tile
            ok = mbar_wait(bar(b_rdone + pb), (jt >> 1) & 1, abort_flag, status);
            QMLA_TR(6);
            if (ok)
              for (int t = 0; t < nrope; ++t) {
                uint32_t idx = tbase + t;
                if (idx >= nslot) idx -= nslot;
                mbar_arrive(bar(b_empty + idx));
              }
          }
          if (ok) ok = mbar_wait(bar(b_pfull + pb), (jt >> 1) & 1, abort_flag, status);
          QMLA_TR(7);
          if (ok && k == k0 && sidx > 0)
            ok = mbar_wait(bar(b_ofree), (sidx - 1) & 1, abort_flag, status);
          if (ok) {
            tc_fence_after();
            // B = P^T (K = tokens, N = heads), MN-major, no swizzle: core matrix =
            //   8 tokens x 16 bytes; SBO = head-block stride, LBO = token-group stride
            const uint64_t bd0 = make_sdesc(pbuf + pb * a.p_bytes, 16 * NPV, 128, 0);
            // A = V^T (M = 128 dims, K = tokens), MN-major, 128-byte swizzle:
            //   LBO = stride between 64-dim halves (bf16), SBO = 8-token group stride
            uint64_t ad0[NB];
            uint32_t vidx[NB];
#pragma unroll
            for (int blk = 0; blk < NB; ++blk) {
              uint32_t idx = tbase + nrope + blk;
              if (idx >= nslot) idx -= nslot;
              vidx[blk] = idx;
              ad0[blk] = make_sdesc(ring + idx * kSlotBytes, 8192, 1024, 2);
            }
#pragma unroll
            for (int ks = 0; ks < kPvSteps; ++ks) {
              // blocks inner: consecutive MMAs go to different accumulators
#pragma unroll
              for (int blk = 0; blk < NB; ++blk) {
                const uint32_t d_o = tmem_base + col_o + blk * OW;
                const uint64_t ad = ad0[blk] + (uint64_t)(ks * (kPvAStep >> 4));
                const uint64_t bd = bd0 + (uint64_t)(ks * (kPvBStep >> 4));
                const uint32_t acc = (k == k0 && ks == 0) ? 0u : 1u;
                if constexpr (FP8)
                  tc_mma_f8_ss(d_o, ad, bd, idesc, acc);
                else
                  tc_mma_f16_ss(d_o, ad, bd, idesc, acc);
              }
            }
#pragma unroll
            for (int blk = 0; blk < NB; ++blk) tc_commit(bar(b_empty + vidx[blk]));
            tc_commit(bar(b_odone + pb));
            QMLA_TR(8);
          }
        }
        tbase += a.n_slot_tile;
        if (tbase >= nslot) tbase -= nslot;
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      ++sidx;
    }
    if (lane == 0 && jt > 0) {
      tc_commit(bar(b_fin + 1));
      volatile int never = 0;
      mbar_wait(bar(b_fin + 1), 0, &never, nullptr, 100000000ull);
    }
  } else if (FP8 && warp == kWarpFix) {
    // ====================================================== FP8 rms fix-up
    uint8_t* rmsbuf = smem + a.off_rms;
    const int qk = a.qk_dim;
    const int zero_end = a.n_qk_slots * 128;  // MMA K boundary (bytes)
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0;
    bool ok = true;
    while (ok && a.fix_slot0 >= 0 && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const uint32_t rb = jt & 1;
        if (lane == 0 && jt >= 2)
          ok = mbar_wait(bar(b_rempty + rb), ((jt - 2) >> 1) & 1, abort_flag, status);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        for (int s = a.fix_slot0; s < a.n_slot_tile && ok; ++s) {
          uint32_t it = jt * a.n_slot_tile + pos_of(s);
          if (lane == 0) ok = mbar_wait(bar(b_full + it % nslot), (it / nslot) & 1, abort_flag, status);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          uint8_t* sl = smem + a.off_ring + (it % nslot) * kSlotBytes;
          const int s0 = s * 128;
          // rms bytes of this slot -> staging[row][b - rms_offset]
          const int lo = max(a.rms_offset, s0), hi = min(a.rms_offset + a.rms_bytes, s0 + 128);
          for (int r = lane; r < kTile; r += 32) {
            for (int b = lo; b < hi; ++b) {
              int off = b - s0;
              rmsbuf[rb * (kTile * 64) + r * 64 + (b - a.rms_offset)] =
                  sl[r * 128 + ((((off >> 4) ^ (r & 7))) << 4) + (off & 15)];
            }
          }
          __syncwarp();
          // bytes in [qk, zero_end) of this slot would meet the MMA: zero them
          const int zlo = max(qk, s0), zhi = min(zero_end, s0 + 128);
          for (int r = lane; r < kTile; r += 32)
            for (int b = zlo; b < zhi; ++b) {
              int off = b - s0;
              sl[r * 128 + ((((off >> 4) ^ (r & 7))) << 4) + (off & 15)] = 0;
            }
          if (s >= a.n_qk_slots) {  // rms-only slot: nothing else reads it
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(b_empty + it % nslot));
          }
        }
        if (!ok) break;
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(b_fix + rb));
      }
    }
  } else if (warp < kSoftmaxWarps) {
    // ====================================================== softmax / epilogue
    const int tid = threadIdx.x;  // 0..255
    const int sp = warp & 3;      // TMEM sub-partition
    const int hw = warp >> 2;     // head half
    const int cpar = (lane >> 1) & 1;
    const int tt = sp * 16 + 8 * (lane & 1) + (lane >> 2);  // token of the tile
    const int H = a.H;
    constexpr int nqk = NQK;
    constexpr int nj = NJ;
    const uint32_t lane_base = (uint32_t)(sp * 32) << 16;
    int head[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) head[j] = hw * (nqk >> 1) + 2 * j + cpar;
    // n-space (P^T / O^T column) of this thread's j-th head
    auto ncol = [&](int j) { return hw * (NPV / 2) + cpar * (NPV / 4) + j; };
    auto head_of_n = [&](int n) -> int {
      int h2 = n / (NPV / 2), c2 = (n % (NPV / 2)) / (NPV / 4), j2 = n % (NPV / 4);
      if (j2 >= nj) return -1;
      int h = h2 * (nqk >> 1) + 2 * j2 + c2;
      return h < H ? h : -1;
    };
    const float kscale = (FP8 && a.k_scale) ? __ldg(a.k_scale) : 1.0f;
    const bool cap = a.logit_cap > 0.f;
    float m_ref[NJ], l_part[NJ], gs[NJ];
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    uint32_t jt = 0, sidx = 0;
    bool ok = true;
    const uint8_t* rmsbuf = smem + a.off_rms;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      int L = __ldg(a.seq_lens + row);
      L = L < 0 ? 0 : L;
      // ---------------- stage Q (the previous segment's QK is complete)
      if constexpr (!FP8) {
        const int upr = a.n_sub_qk * 8;  // 16-byte units (8 elements) per head row
        for (int i = tid; i < nqk * upr; i += kSoftmaxThreads) {
          const int h = i / upr, u = i - h * upr, d0 = u * 8;
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          if (h < H && d0 < a.qk_dim) {
            const bool lat = d0 < a.rank;
            const uint8_t* src = lat ? a.q + ((int64_t)row * a.q_sr + (int64_t)h * a.q_sh + d0) * 2
                                     : a.q_pe + ((int64_t)row * a.qpe_sr + (int64_t)h * a.qpe_sh +
                                                 (d0 - a.rank)) * 2;
            if ((lat ? a.q_vec : a.qpe_vec) && d0 + 8 <= a.qk_dim && a.q_dtype == 0) {
              uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
              w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (d0 + e < a.qk_dim) {
                  uint16_t bits = __bfloat16_as_ushort(
                      __float2bfloat16_rn(load_as_float(src + 2 * e, a.q_dtype)));
                  w[e >> 1] |= (uint32_t)bits << ((e & 1) * 16);
                }
              }
            }
          }
          st_shared_v4(sw128(qbuf + (u >> 3) * a.q_chunk_bytes, h, u & 7), w[0], w[1], w[2], w[3]);
        }
      } else {
        // per-head scale so q*scale spans e4m3's range, then hi/lo split
        for (int h = warp; h < H; h += kSoftmaxWarps) {
          float mx = 0.f;
          for (int d = lane; d < a.qk_dim; d += 32) {
            const uint8_t* src = d < a.rank
                ? a.q + ((int64_t)row * a.q_sr + (int64_t)h * a.q_sh + d) * 2
                : a.q_pe + ((int64_t)row * a.qpe_sr + (int64_t)h * a.qpe_sh + (d - a.rank)) * 2;
            mx = fmaxf(mx, fabsf(load_as_float(src, a.q_dtype)));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          if (lane == 0) hv[96 + h] = mx > 0.f ? 448.f / mx : 1.f;
        }
        named_bar_sync(kBarSoftmax, kSoftmaxThreads);
        const int upr = a.n_sub_qk * 8;  // 16-byte units (16 e4m3) per Q row
        for (int i = tid; i < 2 * nqk * upr; i += kSoftmaxThreads) {
          const int r = i / upr, u = i - r * upr, d0 = u * 16;
          const int h = r < nqk ? r : r - nqk;
          const bool lo_row = r >= nqk;
          uint32_t w[4] = {0u, 0u, 0u, 0u};
          if (h < H) {
            const float sc = hv[96 + h];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int d = d0 + e;
              uint8_t b = 0;
              if (d < a.qk_dim) {
                const uint8_t* src = d < a.rank
                    ? a.q + ((int64_t)row * a.q_sr + (int64_t)h * a.q_sh + d) * 2
                    : a.q_pe + ((int64_t)row * a.qpe_sr + (int64_t)h * a.qpe_sh + (d - a.rank)) * 2;
                const float x = load_as_float(src, a.q_dtype) * sc;
                const uint8_t hi = f32_to_e4m3(x);
                b = lo_row ? f32_to_e4m3(x - e4m3_to_f32(hi)) : hi;
              }
              w[e >> 2] |= (uint32_t)b << ((e & 3) * 8);
            }
          }
          st_shared_v4(sw128(qbuf + (u >> 3) * a.q_chunk_bytes, r, u & 7), w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(kBarSoftmax, kSoftmaxThreads);
      if (lane == 0) mbar_arrive(bar(b_qfull));
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        m_ref[j] = -INFINITY;
        l_part[j] = 0.f;
        float g = a.sm_scale;
        if constexpr (FP8) g *= kscale / (head[j] < H ? hv[96 + head[j]] : 1.f);
        gs[j] = g;
      }

      // ---------------- tiles
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const uint32_t sb = jt % SB;   // S buffer
        const uint32_t pb = jt & 1;    // P buffer / odone / rdone parity
        const int nvalid = min(kTile, L - k * kTile);
        const bool valid = tt < nvalid;
        const uint32_t tbase = (jt * a.n_slot_tile) % nslot;  // ring index of this tile's first slot
        float x[NJ];
        ok = mbar_wait(bar(b_sfull + sb), (jt / SB) & 1, abort_flag, status);
        if (!ok) break;
        if (tid == 0) QMLA_TR(9);
        tc_fence_after();
        {
          const uint32_t tb = tmem_base + lane_base + col_s + sb * SW + hw * (nqk >> 1);
          // S = sum of the KP partials (and of the hi / lo halves for FP8)
          float xp[KP * (FP8 ? 2 : 1)][NJ];
#pragma unroll
          for (int p = 0; p < KP; ++p) {
            load_s_pairs<NJ>(tb + p * SWP, xp[p * (FP8 ? 2 : 1)]);
            if constexpr (FP8) load_s_pairs<NJ>(tb + p * SWP + nqk, xp[p * 2 + 1]);
          }
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            float v = 0.f;
#pragma unroll
            for (int p = 0; p < KP * (FP8 ? 2 : 1); ++p) v += xp[p][j];
            x[j] = v;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(b_sempty + sb));
        // ---- rms divisor -> per-(token, head) factor
        float f[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) f[j] = gs[j];
        if (a.rms_mode != 0) {
          if constexpr (!FP8) {
            if (valid) {
#pragma unroll
              for (int j = 0; j < NJ; ++j) {
                if (j < nj && head[j] < H) {
                  const int d = a.rms_offset + head[j];
                  const int s = d >> 7, e = d & 127;
                  const uint32_t sl = slot_at(tbase, pos_of(s)) + (e >> 6) * 8192;
                  uint16_t bits;
                  asm volatile("ld.shared.u16 %0, [%1];"
                               : "=h"(bits)
                               : "r"(sw128(sl, tt, (e & 63) >> 3) + (e & 7) * 2));
                  const float r = __bfloat162float(__ushort_as_bfloat16(bits));
                  f[j] = r > 0.f ? __fdividef(gs[j], r) : gs[j];
                }
              }
            }
          } else {
            ok = mbar_wait(bar(b_fix + pb), (jt >> 1) & 1, abort_flag, status);
            if (!ok) break;
            if (valid) {
              const uint8_t* rp = rmsbuf + pb * (kTile * 64) + tt * 64;
#pragma unroll
              for (int j = 0; j < NJ; ++j) {
                if (j < nj && head[j] < H) {
                  const int h = head[j];
                  if (a.rms_mode == 3) {
                    // 1 / rms = 2^(3 - code * 6/255)
                    f[j] = gs[j] * exp2f(3.0f - (float)rp[h] * (6.0f / 255.0f));
                  } else {
                    float r;
                    if (a.rms_mode == 2)
                      r = __bfloat162float(__ushort_as_bfloat16(
                          (uint16_t)rp[2 * h] | ((uint16_t)rp[2 * h + 1] << 8)));
                    else
                      r = e4m3_to_f32(rp[h]) * kscale;
                    f[j] = r > 0.f ? __fdividef(gs[j], r) : gs[j];
                  }
                }
              }
            }
          }
        }
        if constexpr (FP8) {
          // the fix-up may stage the next-but-one tile only after this one is consumed
          if (a.fix_slot0 >= 0) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(b_rempty + pb));
          }
        }
        // PV(jt-2) must be done before P buffer sb is rewritten; waiting here also
        // keeps the rms-released signal below at most one phase ahead of its reader
        if (jt >= 2) {
          const uint32_t jp = jt - 2;
          ok = mbar_wait(bar(b_odone + (jp & 1)), (jp >> 1) & 1, abort_flag, status);
          if (!ok) break;
        }
        if constexpr (!FP8) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(b_rdone + pb));
        }
        if (tid == 0) QMLA_TR(10);
        // ---- logits (log2 units) and the lazy-rescale test
        bool need = false;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          float v = -INFINITY;
          if (valid && j < nj && head[j] < H) {
            float s = x[j] * f[j];
            if (cap) s = a.logit_cap * tanhf(s / a.logit_cap);
            v = s * kLog2e;
          }
          x[j] = v;
          need |= v > m_ref[j] + kRescaleThreshold;
        }
        need = named_bar_or(kBarSoftmax, kSoftmaxThreads, need);
        if (tid == 0) QMLA_TR(11);
        if (need) {
          // exact tile max per head: over this warp's 16 tokens, then the 4 sub-partitions
          float wm[NJ];
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            float v = x[j];
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
            v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
            wm[j] = v;
          }
          if (lane < 4 && (lane & 1) == 0) {
#pragma unroll
            for (int j = 0; j < NJ; ++j) red[(hw * 4 + sp) * 32 + 2 * j + cpar] = wm[j];
          }
          named_bar_sync(kBarSoftmax, kSoftmaxThreads);
          bool any_scale = false;
          float alpha[NJ];
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const int c2 = 2 * j + cpar;
            float t = fmaxf(fmaxf(red[(hw * 4 + 0) * 32 + c2], red[(hw * 4 + 1) * 32 + c2]),
                            fmaxf(red[(hw * 4 + 2) * 32 + c2], red[(hw * 4 + 3) * 32 + c2]));
            float mn = fmaxf(m_ref[j], t);
            float al = (mn == -INFINITY) ? 1.f : (m_ref[j] == -INFINITY ? 0.f : exp2f(m_ref[j] - mn));
            alpha[j] = al;
            any_scale |= (al != 1.f) && (k > k0);
            m_ref[j] = mn;
            l_part[j] *= al;
          }
          any_scale = named_bar_or(kBarSoftmax, kSoftmaxThreads, any_scale);  // red[] free again
          if (any_scale) {
            // O holds tiles k0..k-1: wait for PV(k-1), then rescale it in TMEM
            if (sp == 0 && lane < 4 && (lane & 1) == 0) {
#pragma unroll
              for (int j = 0; j < NJ; ++j)
                if (j < nj) hv[head[j] & 31] = alpha[j];
            }
            named_bar_sync(kBarSoftmax, kSoftmaxThreads);
            const uint32_t jp = jt - 1;
            ok = mbar_wait(bar(b_odone + (jp & 1)), (jp >> 1) & 1, abort_flag, status);
            if (!ok) break;
            tc_fence_after();
            float an[NPV / 2];
#pragma unroll
            for (int i = 0; i < NPV / 2; ++i) {
              int h = head_of_n(hw * (NPV / 2) + i);
              an[i] = h >= 0 ? hv[h] : 1.f;
            }
            for (int blk = 0; blk < NB; ++blk) {
#pragma unroll
              for (int part = 0; part < (FP8 ? 2 : 1); ++part) {
                const uint32_t ta = tmem_base + lane_base + col_o + blk * OW + part * NPV + hw * (NPV / 2);
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
            }
            tmem_wait_st();
            named_bar_sync(kBarSoftmax, kSoftmaxThreads);  // hv[] free again
          }
        }
        // ---- P = 2^(x - m) -> P^T buffer sb
        {
          float p[NJP];
#pragma unroll
          for (int j = 0; j < NJP; ++j) {
            if (j < NJ) {
              p[j] = (x[j] == -INFINITY) ? 0.f : ex2_approx(x[j] - m_ref[j]);
              l_part[j] += p[j];
            } else {
              p[j] = 0.f;  // padding columns of P^T
            }
          }
          const uint32_t prow = pbuf + pb * a.p_bytes + (tt >> 3) * (16 * NPV) + (tt & 7) * 16;
          const int n0 = ncol(0);
          if constexpr (!FP8) {
            uint32_t w[NJP / 2];
#pragma unroll
            for (int j = 0; j < NJP; j += 2)
              w[j / 2] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p[j])) |
                         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(p[j + 1])) << 16);
            const uint32_t addr = prow + (n0 >> 3) * 128 + (n0 & 7) * 2;
            if constexpr (NJP == 8)
              st_shared_v4(addr, w[0], w[1], w[2], w[3]);
            else
              st_shared_v2(addr, w[0], w[1]);
          } else {
            uint32_t whi[NJP / 4], wlo[NJP / 4];
#pragma unroll
            for (int q4 = 0; q4 < NJP / 4; ++q4) {
              whi[q4] = 0u;
              wlo[q4] = 0u;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float v = p[q4 * 4 + e];
                const uint8_t hi = f32_to_e4m3(v);
                const uint8_t lo = f32_to_e4m3(v - e4m3_to_f32(hi));
                whi[q4] |= (uint32_t)hi << (8 * e);
                wlo[q4] |= (uint32_t)lo << (8 * e);
              }
            }
            const uint32_t ah = prow + (n0 >> 4) * 128 + (n0 & 15);
            const uint32_t al = prow + ((NPV + n0) >> 4) * 128 + ((NPV + n0) & 15);
            if constexpr (NJP == 8) {
              st_shared_v2(ah, whi[0], whi[1]);
              st_shared_v2(al, wlo[0], wlo[1]);
            } else {
              st_shared_u32(ah, whi[0]);
              st_shared_u32(al, wlo[0]);
            }
          }
          // tokens past the row end: zero their latent rows so P.V stays finite
          if (!valid) {
            constexpr int upr = kSlotBytes / kTile / 16;  // 16-byte units per token per slot
            const int q4 = 2 * hw + cpar;
            for (int i = q4; i < NB * upr; i += 4) {
              const int blk = i / upr, u = i - blk * upr;
              const uint32_t base = slot_at(tbase, nrope + blk) + (u >> 3) * 8192 + tt * 128 + (u & 7) * 16;
              st_shared_v4(base, 0u, 0u, 0u, 0u);
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (tid == 0) QMLA_TR(12);
        if (lane == 0) mbar_arrive(bar(b_pfull + pb));
      }
      if (!ok) break;

      // ---------------- epilogue: O^T / l -> output (or partial)
      {
        const uint32_t jl = jt - 1;
        ok = mbar_wait(bar(b_odone + (jl & 1)), (jl >> 1) & 1, abort_flag, status);
        if (!ok) break;
        tc_fence_after();
        float ls[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          float v = l_part[j];
          v += __shfl_xor_sync(0xffffffffu, v, 1);
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          ls[j] = v;
        }
        if (lane < 4 && (lane & 1) == 0) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) red[(hw * 4 + sp) * 32 + 2 * j + cpar] = ls[j];
        }
        named_bar_sync(kBarSoftmax, kSoftmaxThreads);
        if (sp == 0 && lane < 4 && (lane & 1) == 0) {
#pragma unroll
          for (int j = 0; j < NJ; ++j) {
            const int c2 = 2 * j + cpar;
            if (j < nj && head[j] < H) {
              float lt = red[(hw * 4 + 0) * 32 + c2] + red[(hw * 4 + 1) * 32 + c2] +
                         red[(hw * 4 + 2) * 32 + c2] + red[(hw * 4 + 3) * 32 + c2];
              hv[32 + head[j]] = lt;
              hv[64 + head[j]] = m_ref[j];
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
          float lt = hn[i] >= 0 ? hv[32 + hn[i]] : 0.f;
          linv[i] = lt > 0.f ? oscale / lt : 0.f;
        }
        for (int blk = 0; blk < NB; ++blk) {
          const int d = blk * 128 + sp * 32 + lane;
          const uint32_t ta = tmem_base + lane_base + col_o + blk * OW + hw * (NPV / 2);
          float ov[NPV / 2];
          if constexpr (NPV == 32) {
            tmem_ld16(ta, ov);
            if constexpr (FP8) {
              float ol[16];
              tmem_ld16(ta + NPV, ol);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) ov[i] += ol[i];
            } else {
              tmem_wait_ld();
            }
          } else {
            tmem_ld8(ta, ov);
            if constexpr (FP8) {
              float ol[8];
              tmem_ld8(ta + NPV, ol);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 8; ++i) ov[i] += ol[i];
            } else {
              tmem_wait_ld();
            }
          }
#pragma unroll
          for (int i = 0; i < NPV / 2; ++i) {
            const int h = hn[i];
            if (h >= 0) {
              const float v = ov[i] * linv[i];
              if (full)
                store_from_float(a.o + ((int64_t)row * a.o_sr + (int64_t)h * a.o_sh + d) *
                                           dt_size(a.o_dtype),
                                 a.o_dtype, v);
              else
                a.part_o[((int64_t)slot * H + h) * a.rank + d] = v;
            }
          }
        }
        if (tid < H) {
          const float lt = hv[32 + tid];
          const float l2 = hv[64 + tid] + log2f(lt);  // log2-domain LSE
          if (full) {
            if (a.lse)
              store_from_float(a.lse + ((int64_t)row * a.lse_sr + tid) * dt_size(a.lse_dtype),
                               a.lse_dtype, l2 * kLn2);
          } else {
            a.part_lse[(int64_t)slot * H + tid] = l2;
          }
        }
        tc_fence_before();
        named_bar_sync(kBarSoftmax, kSoftmaxThreads);  // hv[] reads done; O reads done
        if (lane == 0) mbar_arrive(bar(b_ofree));
      }
      ++sidx;
    }
  }
  // ------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kWarpQK) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace qmla
