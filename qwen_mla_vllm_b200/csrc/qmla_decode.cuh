// Paged latent-KV MLA decode for B200 (sm_100a).
//
// One persistent CTA per SM walks a balanced, contiguous range of 64-token
// tiles over all decode rows.  Warp roles:
//   warps 0-3  softmax / epilogue (TMEM sub-partitions 0-3)
//   warp  4    TMA producer: page-table lookups + 3-D tiled bulk loads
//   warp  5    MMA issuer + TMEM owner
//   warps 6-9  (FP8 cache only) e4m3 -> f16 converters
// Per tile:
//   S^T[64 tok, NQK heads] = K_tile[64 x qk] . Q^T      (tcgen05, M=64, K-major)
//   softmax over tokens with the per-(token, head) rms divisor, lazy rescale
//   O^T[rank, NPV]        += V^T[rank x 64] . P^T        (tcgen05, M=128, MN-major)
// The latent part of a tile stays in shared memory from QK until PV, so every
// cache byte crosses HBM once.  Semantics follow the reference Triton kernel
// qwen_mla/ops/mla_decode_attention.py:297-586 (scores, rms divide, softmax,
// split merge) and its stage 2 at :1064-1137.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "qmla_ptx.cuh"

namespace qmla {

constexpr int kTile = 64;             // tokens per tile
constexpr int kSubBytes = 8192;       // 64 rows x 128 B (one 128-byte swizzle column)
constexpr int kSlotBytes = 16384;     // 128 dims of a 16-bit tile = 2 sub-chunks
constexpr int kLandBytes = 8192;      // 128 dims of an FP8 tile
constexpr int kMaxQkChunks = 16;      // QK width <= 1024 elements
constexpr int kMaxCtas = 160;         // persistent CTAs per launch (B200: 148 SMs)
constexpr int kNumSoftmaxThreads = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: P may reach 2^8 before O is rescaled

struct DecodeArgs {
  // query
  const uint8_t* q;
  const uint8_t* q_pe;
  int64_t q_sr, q_sh, qpe_sr, qpe_sh;  // element strides
  int q_dtype;
  // cache addressing for direct (non-TMA) reads: unused by the kernel, kept for tests
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* seq_lens;
  int64_t kv_num_pages;
  int page_size;
  int run_rows;  // gcd(page_size, 64): tokens per TMA box
  // geometry
  int num_rows, H, rank, qk_dim, rms_offset, rms_mode;
  int nqk;           // heads rounded up to a multiple of 8 (QK MMA N)
  int n_sub_qk;      // 64-wide 16-bit sub-chunks covering the QK width (and bf16 rms tail)
  int n_slot_tile;   // MMA-ring slots per tile = ceil(n_sub_qk / 2)
  int n_land_tile;   // FP8 landing slots per tile (covers qk + rms bytes)
  int rms_slot;      // bf16: MMA-ring slot holding the rms tail
  float score_scale; // sm_scale * (k_scale folded on device for FP8)
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
  uint32_t off_ring, nslot, off_q, q_chunk_bytes, off_p, p_bytes, off_land, nland, off_rms,
      off_misc;
};

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

// 16-bit value bits of `v` for the MMA operand type (bf16 for a bf16 cache, f16 for FP8).
template <bool FP8>
__device__ __forceinline__ uint16_t to_op16(float v) {
  if constexpr (FP8) {
    return __half_as_ushort(__float2half_rn(v));
  } else {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
}

// Segment iterator: the CTA's tile range [lo, hi) cut by row boundaries.
struct SegCursor {
  int row, lo, hi;
};
__device__ __forceinline__ int first_row_at(const int32_t* prefix, int n, int t) {
  // largest r with prefix[r] <= t (prefix non-decreasing, prefix[n] > t)
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
// Fetch the next segment; returns false when the range is exhausted.
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

// Byte address (shared window) of element (row r, 16B-unit u) inside a
// 128-byte-swizzled block whose base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128(uint32_t base, int r, int u) {
  return base + (uint32_t)(r * 128 + ((u ^ (r & 7)) << 4));
}

// ---------------------------------------------------------------- the kernel
template <bool FP8, int NB, int NPV>
__global__ void __launch_bounds__(FP8 ? 320 : 192, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeArgs a) {
  constexpr uint32_t kTmemCols = (NB * NPV + 2 * NPV) <= 32    ? 32
                                 : (NB * NPV + 2 * NPV) <= 64  ? 64
                                 : (NB * NPV + 2 * NPV) <= 128 ? 128
                                 : (NB * NPV + 2 * NPV) <= 256 ? 256
                                                               : 512;
  static_assert(NB * NPV + 2 * NPV <= 512, "TMEM budget");
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

  // ------------------------------------------------ shared-memory map
  // misc area: barriers then scratch
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_misc);
  const uint32_t nslot = a.nslot;
  const uint32_t nland = a.nland;
  // barrier indices
  const uint32_t b_full = 0;               // [nslot]
  const uint32_t b_empty = b_full + nslot; // [nslot]
  const uint32_t b_lfull = b_empty + nslot;    // [nland]
  const uint32_t b_lempty = b_lfull + nland;   // [nland]
  const uint32_t b_sfull = b_lempty + nland;   // [2]
  const uint32_t b_sempty = b_sfull + 2;       // [2]
  const uint32_t b_pfull = b_sempty + 2;       // [2]
  const uint32_t b_odone = b_pfull + 2;        // [2]
  const uint32_t b_qfull = b_odone + 2;        // [1]
  const uint32_t b_ofree = b_qfull + 1;        // [1]
  const uint32_t b_rfull = b_ofree + 1;        // [2] FP8 rms tail staged
  const uint32_t b_rempty = b_rfull + 2;       // [2]
  const uint32_t b_fin = b_rempty + 2;          // [1] MMA drain at teardown
  const uint32_t n_bars = b_fin + 1;
  auto bar = [&](uint32_t i) -> uint32_t { return smem_u32(bars + i); };
  uint8_t* misc2 = smem + a.off_misc + ((n_bars * 8 + 15) / 16) * 16;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(misc2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc2 + 4);
  float* red = reinterpret_cast<float*>(misc2 + 16);  // [4][32] per-warp partial maxima/sums

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < nslot; ++i) {
      mbar_init(bar(b_full + i), FP8 ? 4 : 1);
      mbar_init(bar(b_empty + i), 1);
    }
    for (uint32_t i = 0; i < nland; ++i) {
      mbar_init(bar(b_lfull + i), 1);
      mbar_init(bar(b_lempty + i), 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(b_sfull + i), 1);
      mbar_init(bar(b_sempty + i), 1);
      mbar_init(bar(b_pfull + i), 1);
      mbar_init(bar(b_odone + i), 1);
      mbar_init(bar(b_rfull + i), 4);
      mbar_init(bar(b_rempty + i), 1);
    }
    mbar_init(bar(b_qfull), 1);
    mbar_init(bar(b_ofree), 1);
    mbar_init(bar(b_fin), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) prefetch_tmap(&tmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t col_o = 0;
  const uint32_t col_s = NB * NPV;  // two S buffers of NPV columns each

  const uint32_t ring = sbase + a.off_ring;
  const uint32_t qbuf = sbase + a.off_q;
  const uint32_t pbuf = sbase + a.off_p;
  const uint32_t land = sbase + a.off_land;
  int* status = a.status;

  if (warp == 4) {
    // ====================================================== TMA producer
    const uint64_t pol = policy_evict_first();
    const int runs = kTile / a.run_rows;  // <= 4
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    int jt = 0;
    uint32_t armed_m = 0, armed_l = 0;  // slots whose loads were issued
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      int L = __ldg(a.seq_lens + row);
      L = L < 0 ? 0 : L;
      const int32_t* bt = a.block_table + (int64_t)row * a.bt_stride;
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        // page ids of this tile's runs (lane i -> run i)
        int page = -1, y = 0;
        if (lane < runs) {
          int tok0 = k * kTile + lane * a.run_rows;
          if (tok0 < L) {
            page = __ldg(bt + tok0 / a.page_size);
            y = tok0 % a.page_size;
          }
        }
        int pages[4], ys[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          pages[r] = __shfl_sync(0xffffffffu, page, r);
          ys[r] = __shfl_sync(0xffffffffu, y, r);
        }
        if constexpr (!FP8) {
          for (int s = 0; s < a.n_slot_tile && ok; ++s) {
            uint32_t it = (uint32_t)jt * a.n_slot_tile + s;
            uint32_t idx = it % nslot, ph = (it / nslot) & 1;
            if (lane == 0) ok = mbar_wait(bar(b_empty + idx), ph ^ 1, abort_flag, status);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            int nsub = min(2, a.n_sub_qk - 2 * s);
            if (lane == 0) {
              mbar_expect_tx(bar(b_full + idx), (uint32_t)(nsub * kSubBytes));
              uint32_t dst0 = ring + idx * kSlotBytes;
              for (int sc = 0; sc < nsub; ++sc)
                for (int r = 0; r < runs; ++r)
                  tma_load_3d(dst0 + sc * kSubBytes + r * a.run_rows * 128, &tmap,
                              (2 * s + sc) * 64, ys[r], pages[r], bar(b_full + idx), pol);
            }
            armed_m = it + 1;
          }
        } else {
          for (int s = 0; s < a.n_land_tile && ok; ++s) {
            uint32_t it = (uint32_t)jt * a.n_land_tile + s;
            uint32_t idx = it % nland, ph = (it / nland) & 1;
            if (lane == 0) ok = mbar_wait(bar(b_lempty + idx), ph ^ 1, abort_flag, status);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (lane == 0) {
              mbar_expect_tx(bar(b_lfull + idx), (uint32_t)kLandBytes);
              uint32_t dst0 = land + idx * kLandBytes;
              for (int r = 0; r < runs; ++r)
                tma_load_3d(dst0 + r * a.run_rows * 128, &tmap, s * 128, ys[r], pages[r],
                            bar(b_lfull + idx), pol);
            }
            armed_l = it + 1;
          }
        }
      }
    }
    // Teardown after an abort: wait (bounded) until the loads this warp already
    // issued have landed, so no bulk copy still targets shared memory at exit.
    if (!ok && lane == 0) {
      const uint32_t n_armed = FP8 ? armed_l : armed_m;
      const uint32_t ring_n = FP8 ? nland : nslot;
      const uint32_t first = n_armed > ring_n ? n_armed - ring_n : 0u;
      for (uint32_t it = first; it < n_armed; ++it) {
        uint32_t idx = it % ring_n, ph = (it / ring_n) & 1;
        volatile int never = 0;
        mbar_wait(bar((FP8 ? b_lfull : b_full) + idx), ph, &never, nullptr, 20000000ull);
      }
    }
  } else if (warp == 5) {
    // ====================================================== MMA issuer
    const uint32_t fmt = FP8 ? 0u : 1u;
    const uint32_t idesc_qk = make_idesc_f16(fmt, 64, (uint32_t)a.nqk, 0, 0);
    const uint32_t idesc_pv = make_idesc_f16(fmt, 128, NPV, 1, 1);
    const uint32_t q_chunk = a.q_chunk_bytes;
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    int jt = 0, sidx = 0;
    bool ok = true;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      if (lane == 0) ok = mbar_wait(bar(b_qfull), sidx & 1, abort_flag, status);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const int sb = jt & 1;
        if (lane == 0) {
          if (jt >= 2) ok = mbar_wait(bar(b_sempty + sb), ((jt - 2) >> 1) & 1, abort_flag, status);
          tc_fence_after();
          const uint32_t d_s = tmem_base + col_s + sb * NPV;
          int c = 0;  // QK sub-chunk index (64 dims each)
          for (int s = 0; s < a.n_slot_tile && ok; ++s) {
            uint32_t it = (uint32_t)jt * a.n_slot_tile + s;
            uint32_t idx = it % nslot, ph = (it / nslot) & 1;
            ok = mbar_wait(bar(b_full + idx), ph, abort_flag, status);
            if (!ok) break;
            tc_fence_after();
            int nsub = min(2, a.n_sub_qk - 2 * s);
            for (int sc = 0; sc < nsub; ++sc, ++c) {
              uint32_t a_base = ring + idx * kSlotBytes + sc * kSubBytes;
              uint32_t b_base = qbuf + c * q_chunk;
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                uint64_t ad = make_sdesc(a_base + ks * 32, 16, 1024, 2);
                uint64_t bd = make_sdesc(b_base + ks * 32, 16, 1024, 2);
                tc_mma_f16_ss(d_s, ad, bd, idesc_qk, (c | ks) != 0);
              }
            }
            if (FP8 && s >= NB) tc_commit(bar(b_empty + idx));  // rope slot free after QK
          }
          if (ok) tc_commit(bar(b_sfull + sb));
          // ---- PV
          if (ok) ok = mbar_wait(bar(b_pfull + sb), (jt >> 1) & 1, abort_flag, status);
          if (ok && k == k0 && sidx > 0) ok = mbar_wait(bar(b_ofree), (sidx - 1) & 1, abort_flag, status);
          if (ok) {
            tc_fence_after();
            const uint32_t p_base = pbuf + sb * a.p_bytes;
            for (int blk = 0; blk < NB; ++blk) {
              uint32_t it = (uint32_t)jt * a.n_slot_tile + blk;
              uint32_t idx = it % nslot;
              uint32_t v_base = ring + idx * kSlotBytes;
              uint32_t d_o = tmem_base + col_o + blk * NPV;
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                // A = V^T (M = 128 dims, K = 16 tokens), MN-major, 128B swizzle:
                //   LBO = stride between the two 64-dim sub-chunks, SBO = 8-token group stride
                uint64_t ad = make_sdesc(v_base + ks * 2048, kSubBytes, 1024, 2);
                // B = P^T (K = 16 tokens, N = NPV heads), MN-major, no swizzle:
                //   core matrix = 8 tokens x 8 heads; SBO = head-group stride (128 B),
                //   LBO = token-group stride (NPV * 16 B)
                uint64_t bd = make_sdesc(p_base + ks * 2 * NPV * 16, NPV * 16, 128, 0);
                tc_mma_f16_ss(d_o, ad, bd, idesc_pv, !(k == k0 && ks == 0));
              }
            }
            tc_commit(bar(b_odone + sb));
            for (int blk = 0; blk < NB; ++blk) {
              uint32_t it = (uint32_t)jt * a.n_slot_tile + blk;
              tc_commit(bar(b_empty + it % nslot));
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      ++sidx;
    }
    // teardown: every MMA this thread issued must be finished before TMEM is freed
    if (lane == 0 && jt > 0) {
      tc_commit(bar(b_fin));
      volatile int never = 0;
      mbar_wait(bar(b_fin), 0, &never, nullptr, 100000000ull);
    }
  } else if (FP8 && warp >= 6) {
    // ====================================================== FP8 -> f16 converters
    const int ct = threadIdx.x - 192;  // 0..127
    const int crow = ct >> 1;          // token row of the tile
    const int half = ct & 1;           // 64-dim half of the 128-dim slot
    const int rms_bytes = a.rms_mode == 2 ? 2 * a.H : (a.rms_mode == 0 ? 0 : a.H);
    const int qk_bytes = a.qk_dim;
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    int jt = 0;
    bool ok = true;
    uint8_t* rmsbuf = smem + a.off_rms;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      int L = __ldg(a.seq_lens + row);
      L = L < 0 ? 0 : L;
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const int nvalid = min(kTile, L - k * kTile);
        const bool row_ok = crow < nvalid;
        const int rb = jt & 1;
        // the rms staging buffer of this parity must have been read by the softmax
        if (a.rms_mode != 0) {
          if (lane == 0 && jt >= 2)
            ok = mbar_wait(bar(b_rempty + rb), ((jt - 2) >> 1) & 1, abort_flag, status);
          ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        for (int s = 0; s < a.n_land_tile && ok; ++s) {
          uint32_t lit = (uint32_t)jt * a.n_land_tile + s;
          uint32_t lidx = lit % nland, lph = (lit / nland) & 1;
          if (lane == 0) ok = mbar_wait(bar(b_lfull + lidx), lph, abort_flag, status);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          const bool to_mma = s < a.n_slot_tile;
          uint32_t midx = 0;
          if (to_mma) {
            uint32_t it = (uint32_t)jt * a.n_slot_tile + s;
            midx = it % nslot;
            uint32_t ph = (it / nslot) & 1;
            if (lane == 0) ok = mbar_wait(bar(b_empty + midx), ph ^ 1, abort_flag, status);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
          }
          const uint32_t lbase = land + lidx * kLandBytes;
          // rms bytes living in this landing slot -> staging [token][bytes]
          if (a.rms_mode != 0 && half == 0 && row_ok) {
            int b0 = a.rms_offset, b1 = a.rms_offset + rms_bytes;
            int s0 = s * 128, s1 = s0 + 128;
            int lo = max(b0, s0), hi = min(b1, s1);
            const uint8_t* lrow = smem + a.off_land + lidx * kLandBytes;
            for (int b = lo; b < hi; ++b) {
              int off = b - s0;
              int phys = crow * 128 + ((((off >> 4) ^ (crow & 7))) << 4) + (off & 15);
              rmsbuf[rb * (kTile * 64) + crow * 64 + (b - b0)] = lrow[phys];
            }
          }
          if (to_mma) {
            const uint32_t mbase = ring + midx * kSlotBytes + half * kSubBytes;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              // output unit v = dims [8v, 8v+8) of this half -> input bytes 64*half + 8v ..
              int in_byte = 64 * half + 8 * v;
              int gbyte = s * 128 + in_byte;  // byte index in the cache row
              uint32_t w[4] = {0u, 0u, 0u, 0u};
              if (row_ok && gbyte < qk_bytes) {
                uint32_t lo32, hi32;
                uint32_t src = sw128(lbase, crow, in_byte >> 4) + (in_byte & 15);
                asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(lo32), "=r"(hi32) : "r"(src));
                uint32_t bytes[2] = {lo32, hi32};
#pragma unroll
                for (int hw = 0; hw < 4; ++hw) {
                  uint16_t pair = (uint16_t)(bytes[hw >> 1] >> ((hw & 1) * 16));
                  __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)pair, __NV_E4M3);
                  w[hw] = (uint32_t)h2.x | ((uint32_t)h2.y << 16);
                }
                // zero dims at/after the attention width inside this unit
                int rem = qk_bytes - gbyte;
                if (rem < 8) {
#pragma unroll
                  for (int e = 0; e < 8; ++e)
                    if (e >= rem) w[e >> 1] &= (e & 1) ? 0x0000FFFFu : 0xFFFF0000u;
                }
              }
              uint32_t dst = sw128(mbase, crow, v);
              asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]),
                           "r"(w[1]), "r"(w[2]), "r"(w[3])
                           : "memory");
            }
            fence_proxy_async_smem();
          }
          __syncwarp();
          if (lane == 0) {
            if (to_mma) mbar_arrive(bar(b_full + midx));
            mbar_arrive(bar(b_lempty + lidx));
          }
        }
        if (ok && a.rms_mode != 0) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(b_rfull + rb));
        }
      }
    }
  } else if (warp < 4) {
    // ====================================================== softmax / epilogue
    const int tid = threadIdx.x;  // 0..127
    const int H = a.H;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const bool tok_lane = lane < 16;
    const int tt = warp * 16 + lane;  // token of the tile owned by this thread (lane < 16)
    float m_ref[NPV], l_part[NPV];
    const float kscale = (FP8 && a.k_scale) ? __ldg(a.k_scale) : 1.0f;
    const float gscale = a.score_scale * (FP8 ? kscale : 1.0f);
    const bool cap = a.logit_cap > 0.f;
    SegCursor cur{row0, range_lo, range_hi};
    int row, k0, k1, plo, phi;
    int jt = 0, sidx = 0;
    bool ok = true;
    const int q_dt = a.q_dtype;
    const int qes = 2;
    uint8_t* rmsbuf = smem + a.off_rms;
    while (ok && next_segment(a.tile_prefix, cur, row, k0, k1, plo, phi)) {
      int L = __ldg(a.seq_lens + row);
      L = L < 0 ? 0 : L;
      // ---- stage Q (previous segment's QK finished: its last S was consumed)
      {
        const int units_per_row = a.n_sub_qk * 8;  // 16-byte units of 8 elements
        const int total_units = a.nqk * units_per_row;
        for (int i = tid; i < total_units; i += kNumSoftmaxThreads) {
          int h = i / units_per_row;
          int u = i - h * units_per_row;  // unit index along the QK width
          int d0 = u * 8;
          uint32_t wv[4] = {0u, 0u, 0u, 0u};
          if (h < H) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              int d = d0 + e;
              float x = 0.f;
              if (d < a.qk_dim) {
                const uint8_t* src =
                    d < a.rank ? a.q + ((int64_t)row * a.q_sr + (int64_t)h * a.q_sh + d) * qes
                               : a.q_pe + ((int64_t)row * a.qpe_sr + (int64_t)h * a.qpe_sh +
                                           (d - a.rank)) * qes;
                x = load_as_float(src, q_dt);
              }
              uint32_t bits = to_op16<FP8>(x);
              wv[e >> 1] |= bits << ((e & 1) * 16);
            }
          }
          int c = u >> 3;       // 64-dim chunk
          int uc = u & 7;       // unit within the chunk row
          uint32_t dst = sw128(qbuf + c * a.q_chunk_bytes, h, uc);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(wv[0]),
                       "r"(wv[1]), "r"(wv[2]), "r"(wv[3])
                       : "memory");
        }
        fence_proxy_async_smem();
        named_bar_sync(1, kNumSoftmaxThreads);
        if (tid == 0) mbar_arrive(bar(b_qfull));
      }
#pragma unroll
      for (int h = 0; h < NPV; ++h) {
        m_ref[h] = -INFINITY;
        l_part[h] = 0.f;
      }
      for (int k = k0; k < k1 && ok; ++k, ++jt) {
        const int sb = jt & 1;
        const int nvalid = min(kTile, L - k * kTile);
        const bool valid = tok_lane && tt < nvalid;
        float x[NPV];
        // ---- scores
        if (tid == 0) ok = mbar_wait(bar(b_sfull + sb), (jt >> 1) & 1, abort_flag, status);
        ok = named_bar_or(1, kNumSoftmaxThreads, !ok) ? false : true;
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int g = 0; g < NPV / 8; ++g) {
          if (g * 8 < a.nqk) tmem_ld8(tmem_base + lane_base + col_s + sb * NPV + g * 8, x + g * 8);
        }
        tmem_wait_ld();
        // ---- rms divisor
        float rinv[NPV];
#pragma unroll
        for (int h = 0; h < NPV; ++h) rinv[h] = 1.f;
        if (a.rms_mode != 0) {
          if constexpr (!FP8) {
            if (valid) {
#pragma unroll
              for (int h = 0; h < NPV; ++h) {
                if (h < H) {
                  const int d = a.rms_offset + h;  // element of the cache row
                  const int s = d >> 7;            // MMA-ring slot of the tile
                  const int e = d & 127;
                  uint32_t it = (uint32_t)jt * a.n_slot_tile + s;
                  uint32_t sl = ring + (it % nslot) * kSlotBytes + (e >> 6) * kSubBytes;
                  uint32_t addr = sw128(sl, tt, (e & 63) >> 3) + (e & 7) * 2;
                  uint16_t bits;
                  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(bits) : "r"(addr));
                  float r = __bfloat162float(__ushort_as_bfloat16(bits));
                  rinv[h] = r > 0.f ? 1.f / r : 1.f;
                }
              }
            }
          } else {
            if (tid == 0) ok = mbar_wait(bar(b_rfull + sb), (jt >> 1) & 1, abort_flag, status);
            ok = named_bar_or(1, kNumSoftmaxThreads, !ok) ? false : true;
            if (!ok) break;
            if (valid) {
              const uint8_t* rp = rmsbuf + sb * (kTile * 64) + tt * 64;
#pragma unroll
              for (int h = 0; h < NPV; ++h) {
                if (h < H) {
                  float r;
                  if (a.rms_mode == 3) {
                    r = exp2f(-3.0f + (float)rp[h] * (6.0f / 255.0f));
                  } else if (a.rms_mode == 2) {
                    uint16_t bits = (uint16_t)rp[2 * h] | ((uint16_t)rp[2 * h + 1] << 8);
                    r = __bfloat162float(__ushort_as_bfloat16(bits));
                  } else {
                    __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)rp[h], __NV_E4M3);
                    r = __half2float(__half(hr)) * kscale;
                  }
                  rinv[h] = r > 0.f ? 1.f / r : 1.f;
                }
              }
            }
          }
        }
        // S and rms consumed: release the S buffer (and rms slot / staging)
        tc_fence_before();
        named_bar_sync(1, kNumSoftmaxThreads);
        if (tid == 0) {
          mbar_arrive(bar(b_sempty + sb));
          if constexpr (!FP8) {
            for (int s = NB; s < a.n_slot_tile; ++s) {
              uint32_t it = (uint32_t)jt * a.n_slot_tile + s;
              mbar_arrive(bar(b_empty + it % nslot));
            }
          } else {
            if (a.rms_mode != 0) mbar_arrive(bar(b_rempty + sb));
          }
        }
        // ---- logits in log2 units
        float wmax[NPV];
#pragma unroll
        for (int h = 0; h < NPV; ++h) {
          float v = -INFINITY;
          if (valid && h < H) {
            float s = x[h] * (gscale * rinv[h]);
            if (cap) s = a.logit_cap * tanhf(s / a.logit_cap);
            v = s * kLog2e;
          }
          x[h] = v;
          wmax[h] = v;
        }
        bool need = false;
#pragma unroll
        for (int h = 0; h < NPV; ++h) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) wmax[h] = fmaxf(wmax[h], __shfl_xor_sync(0xffffffffu, wmax[h], o));
          need |= (h < H) && (wmax[h] > m_ref[h] + kRescaleThreshold);
        }
        need = named_bar_or(1, kNumSoftmaxThreads, need);
        if (need) {
          if (lane == 0) {
#pragma unroll
            for (int h = 0; h < NPV; ++h) red[warp * 32 + h] = wmax[h];
          }
          named_bar_sync(1, kNumSoftmaxThreads);
          float alpha[NPV];
          bool any_scale = false;
#pragma unroll
          for (int h = 0; h < NPV; ++h) {
            float t = fmaxf(fmaxf(red[h], red[32 + h]), fmaxf(red[64 + h], red[96 + h]));
            float mn = fmaxf(m_ref[h], t);
            alpha[h] = (m_ref[h] == -INFINITY) ? 0.f : exp2f(m_ref[h] - mn);
            if (mn == -INFINITY) alpha[h] = 1.f;
            any_scale |= alpha[h] != 1.f;
            m_ref[h] = mn;
          }
          named_bar_sync(1, kNumSoftmaxThreads);  // red[] may be reused
          if (k > k0 && any_scale) {
            // O holds tiles k0..k-1: wait for PV(k-1), then rescale it in TMEM
            const int jp = jt - 1;
            if (tid == 0) ok = mbar_wait(bar(b_odone + (jp & 1)), (jp >> 1) & 1, abort_flag, status);
            ok = named_bar_or(1, kNumSoftmaxThreads, !ok) ? false : true;
            if (!ok) break;
            tc_fence_after();
            for (int blk = 0; blk < NB; ++blk) {
#pragma unroll
              for (int g = 0; g < NPV / 8; ++g) {
                float ov[8];
                uint32_t ta = tmem_base + lane_base + col_o + blk * NPV + g * 8;
                tmem_ld8(ta, ov);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 8; ++e) ov[e] *= alpha[g * 8 + e];
                tmem_st8(ta, ov);
              }
            }
            tmem_wait_st();
          }
#pragma unroll
          for (int h = 0; h < NPV; ++h) l_part[h] *= alpha[h];
        }
        // ---- probabilities -> P^T buffer sb
        if (jt >= 2) {
          const int jp = jt - 2;  // PV(jp) read this P buffer
          if (tid == 0) ok = mbar_wait(bar(b_odone + (jp & 1)), (jp >> 1) & 1, abort_flag, status);
          ok = named_bar_or(1, kNumSoftmaxThreads, !ok) ? false : true;
          if (!ok) break;
        }
        if (tok_lane) {
          uint32_t pw[NPV / 2];
#pragma unroll
          for (int h = 0; h < NPV; h += 2) {
            float p0 = (x[h] == -INFINITY) ? 0.f : exp2f(x[h] - m_ref[h]);
            float p1 = (x[h + 1] == -INFINITY) ? 0.f : exp2f(x[h + 1] - m_ref[h + 1]);
            l_part[h] += p0;
            l_part[h + 1] += p1;
            pw[h / 2] = (uint32_t)to_op16<FP8>(p0) | ((uint32_t)to_op16<FP8>(p1) << 16);
          }
          const uint32_t pb = pbuf + sb * a.p_bytes + (tt >> 3) * (NPV * 16) + (tt & 7) * 16;
#pragma unroll
          for (int g = 0; g < NPV / 8; ++g) {
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(pb + g * 128),
                         "r"(pw[g * 4 + 0]), "r"(pw[g * 4 + 1]), "r"(pw[g * 4 + 2]),
                         "r"(pw[g * 4 + 3])
                         : "memory");
          }
          if constexpr (!FP8) {
            // tokens past the row end: zero their latent rows so P*V stays finite
            if (tt >= nvalid) {
              for (int blk = 0; blk < NB; ++blk) {
                uint32_t it = (uint32_t)jt * a.n_slot_tile + blk;
                uint32_t base = ring + (it % nslot) * kSlotBytes + tt * 128;
#pragma unroll
                for (int sc = 0; sc < 2; ++sc)
#pragma unroll
                  for (int u = 0; u < 8; ++u)
                    asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(
                                     base + sc * kSubBytes + u * 16),
                                 "r"(0u)
                                 : "memory");
              }
            }
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(1, kNumSoftmaxThreads);
        if (tid == 0) mbar_arrive(bar(b_pfull + sb));
      }
      if (!ok) break;
      // ---- epilogue: O^T / l -> output (or partial)
      {
        const int jl = jt - 1;
        if (tid == 0) ok = mbar_wait(bar(b_odone + (jl & 1)), (jl >> 1) & 1, abort_flag, status);
        ok = named_bar_or(1, kNumSoftmaxThreads, !ok) ? false : true;
        if (!ok) break;
        tc_fence_after();
        // total l per head: sum over the 16 token lanes then over the 4 warps
#pragma unroll
        for (int h = 0; h < NPV; ++h) {
          float v = tok_lane ? l_part[h] : 0.f;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          l_part[h] = v;
        }
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < NPV; ++h) red[warp * 32 + h] = l_part[h];
        }
        named_bar_sync(1, kNumSoftmaxThreads);
        float linv[NPV];
#pragma unroll
        for (int h = 0; h < NPV; ++h) {
          float lt = red[h] + red[32 + h] + red[64 + h] + red[96 + h];
          l_part[h] = lt;
          linv[h] = lt > 0.f ? 1.f / lt : 0.f;
        }
        const bool full = (plo >= range_lo) && (phi <= range_hi);
        const int slot = (plo <= range_lo) ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
        const float oscale = FP8 ? kscale : 1.0f;
        for (int blk = 0; blk < NB; ++blk) {
          const int d = blk * 128 + warp * 32 + lane;
#pragma unroll
          for (int g = 0; g < NPV / 8; ++g) {
            float ov[8];
            tmem_ld8(tmem_base + lane_base + col_o + blk * NPV + g * 8, ov);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int h = g * 8 + e;
              if (h < H) {
                float v = ov[e] * linv[h] * oscale;
                if (full) {
                  store_from_float(a.o + ((int64_t)row * a.o_sr + (int64_t)h * a.o_sh + d) *
                                             dt_size(a.o_dtype),
                                   a.o_dtype, v);
                } else {
                  a.part_o[((int64_t)slot * H + h) * a.rank + d] = v;
                }
              }
            }
          }
        }
#pragma unroll
        for (int h = 0; h < NPV; ++h) {
          if (h == tid && h < H) {
            // log2-domain LSE of this segment
            float l2 = m_ref[h] + log2f(l_part[h]);
            if (full) {
              if (a.lse)
                store_from_float(a.lse + ((int64_t)row * a.lse_sr + h) * dt_size(a.lse_dtype),
                                 a.lse_dtype, l2 * kLn2);
            } else {
              a.part_lse[(int64_t)slot * H + h] = l2;
            }
          }
        }
        tc_fence_before();
        named_bar_sync(1, kNumSoftmaxThreads);
        if (tid == 0) mbar_arrive(bar(b_ofree));
      }
      ++sidx;
    }
  }
  // ------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace qmla
