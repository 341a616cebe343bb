// Small kernels around the decode kernel: the work plan (tile prefix), the
// split merge, the DCP correction / merge, and the FP8 cache writer.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "qmla_decode.cuh"
#include "qmla.h"

namespace qmla {

// Exclusive prefix of ceil(max(len,0)/kTile) over the rows, plus the total, the G + 1
// CTA range bounds of the decode kernel's partition (range_bound), and clears the device
// status word.  One block of 1024 threads.  Partition rule shared with the host planner
// (qmla_plan) for the prefix.
// A work row is `fold` consecutive decode rows; its length is the longest of theirs.
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ seq_lens, int n,
                                                    int fold, int32_t* __restrict__ prefix,
                                                    int* __restrict__ status, int G, int seg_cost,
                                                    int32_t* __restrict__ bounds,
                                                    int* __restrict__ row_done) {
  if (row_done)  // per-row piece counters of the decode kernel's in-kernel merge
    for (int i = threadIdx.x; i < n; i += blockDim.x) row_done[i] = 0;
  __shared__ int warp_sums[32];
  __shared__ int carry_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    carry_s = 0;
    prefix[0] = 0;
    if (status) *status = 0;
  }
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    int i = base + tid;
    int v = 0;
    if (i < n) {
      int L = 0;
      for (int d = 0; d < fold; ++d) L = max(L, seq_lens[(int64_t)i * fold + d]);
      v = L > 0 ? (L + kTile - 1) / kTile : 0;
    }
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    int incl = x + (warp > 0 ? warp_sums[warp - 1] : 0) + carry_s;
    if (i < n) prefix[i + 1] = incl;
    __syncthreads();
    if (tid == 1023) carry_s = incl;
    __syncthreads();
  }
  __threadfence_block();
  __syncthreads();  // the prefix is complete (global writes of this block are visible to it)
  for (int c = tid; c <= G; c += blockDim.x) bounds[c] = range_bound(prefix, n, G, seg_cost, c);
}

// The range bounds alone, for a prefix planned on the host (qmla_plan); also clears the
// device status word.  One block.
__global__ void __launch_bounds__(256) bounds_kernel(const int32_t* __restrict__ prefix, int n,
                                                     int* __restrict__ status, int G, int seg_cost,
                                                     int32_t* __restrict__ bounds,
                                                     int* __restrict__ row_done) {
  if (threadIdx.x == 0 && status) *status = 0;
  if (row_done)
    for (int i = threadIdx.x; i < n; i += blockDim.x) row_done[i] = 0;
  for (int c = threadIdx.x; c <= G; c += blockDim.x)
    bounds[c] = range_bound(prefix, n, G, seg_cost, c);
}

// Merge of the per-CTA partial segments of rows that crossed a CTA boundary
// (the reference's stage 2, mla_decode_attention.py:1064-1137, over the
// decode kernel's partition).  One block per (work row, query row); with few rows the output
// dims are also split over gridDim.z blocks of 128.  Rows inside one CTA range are final
// already.  Work rows of length 0 get o = 0 and lse = -inf.  Query row r of work row g is head
// r % H of decode row g * fold + r / H.  The pieces' lse values are read in parallel and each
// thread keeps four partial loads in flight: with a serial walk over the pieces, a config-4 call
// (8 rows cut into 18 pieces each) spent 55 us here, one dependent load at a time.
__global__ void __launch_bounds__(128) split_merge_kernel(const DecodeArgs a) {
  const int row = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const int d0 = blockIdx.z * 128 + tid, dstep = gridDim.z * 128;  // rank is a multiple of 128
  const int plo = __ldg(a.tile_prefix + row), phi = __ldg(a.tile_prefix + row + 1);
  const int R = a.R, D = a.rank;
  const int dq = r / a.H, h = r - dq * a.H;
  const int osz = dt_size(a.o_dtype);
  uint8_t* orow = a.o + (((int64_t)row * a.fold + dq) * a.o_sr + (int64_t)h * a.o_sh) * osz;
  uint8_t* lrow = a.lse ? a.lse + (((int64_t)row * a.fold + dq) * a.lse_sr + h) * dt_size(a.lse_dtype) : nullptr;
  const bool lse_writer = lrow && blockIdx.z == 0 && tid == 0;
  if (phi == plo) {
    for (int d = d0; d < D; d += dstep) store_from_float(orow + d * osz, a.o_dtype, 0.f);
    if (lse_writer) store_from_float(lrow, a.lse_dtype, -INFINITY);
    return;
  }
  // CTA ranges that hold tiles of this row (the decode kernel's partition, range_bounds)
  __shared__ int bnd[kMaxCtas + 1];
  for (int c = tid; c <= a.G; c += blockDim.x) bnd[c] = __ldg(a.range_bounds + c);
  __syncthreads();
  auto cta_of = [&](int t) {  // the non-empty range holding tile t: largest c with bnd[c] <= t
    int lo = 0, hi = a.G;
    while (hi - lo > 1) {
      const int m = (lo + hi) >> 1;
      if (bnd[m] <= t)
        lo = m;
      else
        hi = m;
    }
    return lo;
  };
  const int c0 = cta_of(plo), c1 = cta_of(phi - 1);
  if (c0 == c1) return;  // the row lies inside one CTA range: already final
  __shared__ float wts[kMaxCtas];
  __shared__ int slots[kMaxCtas];
  __shared__ float red[4];
  __shared__ int np_s;
  if (tid == 0) {
    int np = 0;  // empty ranges between c0 and c1 wrote nothing
    for (int c = c0; c <= c1; ++c)
      if (bnd[c] < bnd[c + 1]) slots[np++] = (plo <= bnd[c]) ? 2 * c : 2 * c + 1;
    np_s = np;
  }
  __syncthreads();
  const int np = np_s;
  const int lane = tid & 31, warp = tid >> 5;
  // m = max of the pieces' lse (log2 units), then their weights 2^(lse - m) and the sum
  float m = -INFINITY;
  for (int i = tid; i < np; i += blockDim.x) {
    const float l = __ldg(a.part_lse + (int64_t)slots[i] * R + r);
    wts[i] = l;
    m = fmaxf(m, l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();  // red[] is reused below
  float sum = 0.f;
  for (int i = tid; i < np; i += blockDim.x) {
    const float w = (m == -INFINITY) ? 0.f : exp2f(wts[i] - m);
    wts[i] = w;
    sum += w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red[warp] = sum;
  __syncthreads();
  sum = (red[0] + red[1]) + (red[2] + red[3]);
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  // O = sum_i w_i O_i / sum: four independent partial sums, so four loads are in flight
  const int64_t sstride = (int64_t)R * D;  // floats between consecutive slots
  for (int d = d0; d < D; d += dstep) {
    const float* po = a.part_o + (int64_t)r * D + d;
    float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
    int i = 0;
    for (; i + 4 <= np; i += 4) {
      const float v0 = __ldg(po + slots[i] * sstride), v1 = __ldg(po + slots[i + 1] * sstride);
      const float v2 = __ldg(po + slots[i + 2] * sstride), v3 = __ldg(po + slots[i + 3] * sstride);
      acc0 += wts[i] * v0;
      acc1 += wts[i + 1] * v1;
      acc2 += wts[i + 2] * v2;
      acc3 += wts[i + 3] * v3;
    }
    for (; i < np; ++i) acc0 += wts[i] * __ldg(po + slots[i] * sstride);
    store_from_float(orow + d * osz, a.o_dtype, ((acc0 + acc1) + (acc2 + acc3)) * inv);
  }
  if (lse_writer) store_from_float(lrow, a.lse_dtype, (m + log2f(sum)) * kLn2);
}

// FP8 caches: each work row's Q buffer image for the decode kernel, so that the kernel stages
// Q with plain 16-byte copies.  Query row h (head h % H of decode row g * fold + h / H) is
// scaled by sc = 448 / max|q| to span e4m3's range and split as q * sc = hi + lo in e4m3; hi goes
// to row h and lo to row h + nqk of the 128-byte-swizzled column chunks, exactly as the kernel
// lays out its shared memory; rows past R and columns past qk_dim are zero.  sc goes to
// q_scale[g * nqk + h].  One block of 128 threads per (work row, query row); a thread holds two
// 16-element units (QK width <= 2048), all loaded before any is converted.
__global__ void __launch_bounds__(128) q_fp8_prep_kernel(const DecodeArgs a, int nqk, uint8_t* img,
                                                         float* q_scale) {
  const int g = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int R = a.R, H = a.H;
  const int upr = a.n_sub_qk * 8;  // 16-element units per row
  uint8_t* dst = img + (int64_t)g * a.q_img_bytes;
  float v[2][16];
  float mx = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int u = tid + 128 * k;
#pragma unroll
    for (int e = 0; e < 16; ++e) v[k][e] = 0.f;
    if (h < R && u < upr) {
      const int dq = h / H, hh = h - dq * H;
      const int64_t qrow = (int64_t)g * a.fold + dq;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int d = u * 16 + e;
        if (d < a.qk_dim) {
          const uint8_t* src = d < a.rank ? a.q + ((int64_t)qrow * a.q_sr + (int64_t)hh * a.q_sh + d) * 2
                                          : a.q_pe + ((int64_t)qrow * a.qpe_sr + (int64_t)hh * a.qpe_sh +
                                                      (d - a.rank)) * 2;
          v[k][e] = load_as_float(src, a.q_dtype);
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) mx = fmaxf(mx, fabsf(v[k][e]));
    }
  }
  __shared__ float red[4];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  const float sc = mx > 0.f ? 448.f / mx : 1.f;
  if (tid == 0 && h < R) q_scale[(int64_t)g * nqk + h] = sc;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int u = tid + 128 * k;
    if (u >= upr) continue;
    uint32_t whi[4] = {0u, 0u, 0u, 0u}, wlo[4] = {0u, 0u, 0u, 0u};
    if (h < R && u * 16 < a.qk_dim) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x = v[k][e] * sc;
        const uint8_t hi = f32_to_e4m3(x);
        const uint8_t lo = f32_to_e4m3(x - e4m3_to_f32(hi));
        whi[e >> 2] |= (uint32_t)hi << ((e & 3) * 8);
        wlo[e >> 2] |= (uint32_t)lo << ((e & 3) * 8);
      }
    }
    uint8_t* chunk = dst + (int64_t)(u >> 3) * a.q_chunk_bytes;
    *reinterpret_cast<uint4*>(chunk + sw128(0u, h, u & 7)) = make_uint4(whi[0], whi[1], whi[2], whi[3]);
    *reinterpret_cast<uint4*>(chunk + sw128(0u, h + nqk, u & 7)) = make_uint4(wlo[0], wlo[1], wlo[2], wlo[3]);
  }
}

// DCP output correction for one rank (qwen_mla/dcp_fix.py:31-98): grid (B, H).
__global__ void dcp_correct_kernel(uint8_t* out, int out_dt, int64_t osb, int64_t osh,
                                   const float* lses, int64_t lsn, int64_t lsb, float* lse_out,
                                   int N, int cp_rank, int H, int D, int base_e) {
  const int b = blockIdx.x, h = blockIdx.y;
  __shared__ float factor_s;
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int n = 0; n < N; ++n) {
      float v = lses[n * lsn + b * lsb + h];
      if (v != v || v == INFINITY) v = -INFINITY;
      mx = fmaxf(mx, v);
    }
    float m0 = (mx == -INFINITY) ? 0.f : mx;
    float acc = 0.f;
    for (int n = 0; n < N; ++n) {
      float v = lses[n * lsn + b * lsb + h];
      if (v != v || v == INFINITY) v = -INFINITY;
      acc += base_e ? expf(v - m0) : exp2f(v - m0);
    }
    float g = (base_e ? logf(acc) : log2f(acc)) + m0;
    if (lse_out) lse_out[b * lsb + h] = g;
    float own = lses[cp_rank * lsn + b * lsb + h] - g;
    if (own != own || own == INFINITY) own = -INFINITY;
    factor_s = base_e ? expf(own) : exp2f(own);
  }
  __syncthreads();
  const float f = factor_s;
  const int es = dt_size(out_dt);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    uint8_t* p = out + ((int64_t)b * osb + (int64_t)h * osh + d) * es;
    float v = load_as_float(p, out_dt) * f;
    if (f == 0.f) v = 0.f;
    store_from_float(p, out_dt, v);
  }
}

// Fused merge of N DCP partials: grid (B, H).
__global__ void dcp_merge_kernel(const uint8_t* parts, int parts_dt, const float* part_lse,
                                 uint8_t* o, int o_dt, float* lse, int N, int B, int H, int D) {
  const int b = blockIdx.x, h = blockIdx.y;
  __shared__ float w_s[64];
  if (threadIdx.x == 0) {
    float mx = -INFINITY;
    for (int n = 0; n < N; ++n) {
      float v = part_lse[((int64_t)n * B + b) * H + h];
      if (v != v || v == INFINITY) v = -INFINITY;
      w_s[n] = v;
      mx = fmaxf(mx, v);
    }
    float m0 = (mx == -INFINITY) ? 0.f : mx;
    float acc = 0.f;
    for (int n = 0; n < N; ++n) acc += expf(w_s[n] - m0);
    float g = logf(acc) + m0;
    for (int n = 0; n < N; ++n) {
      const float e = w_s[n] - g;  // NaN when every partial is empty: weight 0, as dcp_fix does
      w_s[n] = (e != e || e == INFINITY) ? 0.f : expf(e);
    }
    if (lse) lse[(int64_t)b * H + h] = g;
  }
  __syncthreads();
  const int pes = dt_size(parts_dt), oes = dt_size(o_dt);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int n = 0; n < N; ++n) {
      float w = w_s[n];
      if (w == 0.f) continue;
      acc += w * load_as_float(parts + ((((int64_t)n * B + b) * H + h) * D + d) * pes, parts_dt);
    }
    store_from_float(o + (((int64_t)b * H + h) * D + d) * oes, o_dt, acc);
  }
}

// FP8 cache row writer (qwen_mla/mla_impl.py:309-342).  grid = n_tokens.
__global__ void fp8_cache_write_kernel(const __nv_bfloat16* latent, int64_t lat_stride,
                                       const __nv_bfloat16* k_pe, int64_t kpe_stride,
                                       const int64_t* slots, int rank, int rope, int heads,
                                       int rms_mode, const float* k_scale, uint8_t* cache,
                                       int64_t row_stride) {
  const int i = blockIdx.x;
  int64_t s = slots[i];
  if (s < 0) s = 0;
  uint8_t* dst = cache + s * row_stride;
  const float inv = 1.0f / (k_scale ? *k_scale : 1.0f);
  for (int d = threadIdx.x; d < rank + rope; d += blockDim.x) {
    float x = d < rank ? __bfloat162float(latent[(int64_t)i * lat_stride + d])
                       : __bfloat162float(k_pe[(int64_t)i * kpe_stride + (d - rank)]);
    float y = fminf(fmaxf(x * inv, -448.f), 448.f);
    dst[d] = (uint8_t)__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
  }
  for (int h = threadIdx.x; h < heads; h += blockDim.x) {
    __nv_bfloat16 rb = k_pe[(int64_t)i * kpe_stride + rope + h];
    if (rms_mode == QMLA_RMS_LOG8) {
      float r = fmaxf(__bfloat162float(rb), 1e-30f);
      float code = (log2f(r) - (-3.0f)) * (255.0f / 6.0f);
      code = fminf(fmaxf(rintf(code), 0.f), 255.f);
      dst[rank + rope + h] = (uint8_t)code;
    } else {
      uint16_t bits = __bfloat16_as_ushort(rb);
      dst[rank + rope + 2 * h] = (uint8_t)(bits & 0xFF);
      dst[rank + rope + 2 * h + 1] = (uint8_t)(bits >> 8);
    }
  }
}

// ---------------------------------------------------------------- prefill context gather
// qwen_mla/ops/mla_gather.py:28-76 (gather_cache_torch).  Destination row j belongs to
// sequence s = token_to_seq[j] and holds its token tok = j - cu_seq_lens[s] (+ seq_starts[s]),
// found in page block_table[s][tok / page_size] at offset tok % page_size.
//   2-byte cache: the whole row (n_copy elements) is copied, converted to the destination type.
//   FP8 cache:    columns [0, n_e4m3) = e4m3 * scale; then rms_heads columns from rms_off
//                 decoded from the log8 code or the raw bf16 bytes; later columns untouched.
// One warp per destination row, 16-byte loads and stores where every row start is aligned.
// Rows whose indices fall outside the tables are skipped and flagged in *status.
struct GatherArgs {
  const uint8_t* src;
  int64_t src_sp, src_st;  // bytes per page / per token
  int page_size, num_pages;
  const int32_t* bt;
  int64_t bt_stride;
  int bt_cols;
  const int32_t* cu;
  const int32_t* t2s;
  const int32_t* starts;
  int num_seqs, num_tokens;
  uint8_t* dst;
  int64_t dst_sr;  // bytes per destination row
  int dst_dt, src_dt;
  int n_copy;                          // 2-byte cache: elements per row
  int n_e4m3;                          // FP8 cache: e4m3 columns
  int rms_off, rms_heads, rms_mode;    // FP8 cache: log8 / bf16-byte tail (rms_heads 0: none)
  const float* scale;
  int* status;
};

constexpr int kGatherWarps = 8;   // warps per block
constexpr int kGatherBatch = 8;   // rows per warp step; lane r < 8 resolves row r's indices
constexpr int kGatherRows = 4;    // rows whose 16-byte loads are in flight together
constexpr int kGatherSlots = 2;   // chunks per lane per row in one pass (64 chunks of 16 B)

// Streaming (evict-first) 16-byte accesses: every cache row is read once, every
// destination row written once.
__device__ __forceinline__ uint4 ld_stream16(const uint8_t* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream16(uint8_t* p, uint4 v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}

// 16 consecutive floats to the destination type, as 16-byte stores.
__device__ __forceinline__ void store16_vec(uint8_t* p, int dt, const float* f) {
  if (dt == QMLA_DT_F32) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
      st_stream16(p + 16 * k, make_uint4(__float_as_uint(f[4 * k]), __float_as_uint(f[4 * k + 1]),
                                         __float_as_uint(f[4 * k + 2]), __float_as_uint(f[4 * k + 3])));
    return;
  }
  uint32_t w[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (dt == QMLA_DT_BF16) {
      __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&b);
    } else {
      __half2 h = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
      w[k] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  st_stream16(p, make_uint4(w[0], w[1], w[2], w[3]));
  st_stream16(p + 16, make_uint4(w[4], w[5], w[6], w[7]));
}

__device__ __forceinline__ float e4m3_to_float(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// 16 e4m3 bytes -> 16 floats, each the exact e4m3 value times sc rounded once to f32.
__device__ __forceinline__ void e4m3x16(const uint4 v, float sc, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(
        (__nv_fp8x2_storage_t)((w[k >> 1] >> (16 * (k & 1))) & 0xFFFFu), __NV_E4M3);
    const float2 x = __half22float2(__half2(hr));
    f[2 * k] = __fmul_rn(x.x, sc);
    f[2 * k + 1] = __fmul_rn(x.y, sc);
  }
}

// Byte offset of destination row j's source row, or -1 when its sequence, token or page
// index falls outside the tables (mla_gather.py:41-47 index arithmetic).
__device__ __forceinline__ int64_t gather_row_offset(const GatherArgs& a, int64_t j) {
  const int s = __ldg(a.t2s + j);
  if (s < 0 || s >= a.num_seqs) return -1;
  const int64_t tok = j - (int64_t)__ldg(a.cu + s) + (a.starts ? (int64_t)__ldg(a.starts + s) : 0);
  if (tok < 0 || tok / a.page_size >= a.bt_cols) return -1;
  const int64_t blk = __ldg(a.bt + (int64_t)s * a.bt_stride + tok / a.page_size);
  if (blk < 0 || blk >= a.num_pages) return -1;
  return blk * a.src_sp + (tok % a.page_size) * a.src_st;
}

// One warp per 8 consecutive destination rows per step: lanes 0..7 resolve the rows' index
// chains in parallel (the next step's chains are resolved while this step's loads are in
// flight), then the 16-byte chunks of 4 rows at a time are loaded before any is stored.
template <bool VEC>
__global__ void __launch_bounds__(32 * kGatherWarps) gather_cache_kernel(const GatherArgs a) {
  const int lane = threadIdx.x & 31;
  const int dsz = a.dst_dt == QMLA_DT_F32 ? 4 : 2;
  const float sc = a.scale ? __ldg(a.scale) : 1.0f;
  const bool fp8 = a.src_dt == QMLA_DT_FP8E4M3;
  const bool same = a.dst_dt == a.src_dt;
  const int unit = fp8 ? 16 : 8;  // columns per 16-byte source chunk
  const int ncols = fp8 ? a.n_e4m3 : a.n_copy;
  const int nchunk = VEC ? ncols / unit : 0;
  const int64_t stride = (int64_t)gridDim.x * kGatherWarps * kGatherBatch;
  int64_t base = ((int64_t)blockIdx.x * kGatherWarps + (threadIdx.x >> 5)) * kGatherBatch;
  auto resolve = [&](int64_t b) -> int64_t {
    int64_t off = -1;
    if (lane < kGatherBatch && b + lane < a.num_tokens) {
      off = gather_row_offset(a, b + lane);
      if (off < 0 && a.status) atomicOr(a.status, QMLA_DEV_ERR_INDEX);
    }
    return off;
  };
  int64_t my = base < a.num_tokens ? resolve(base) : -1;
  for (; base < a.num_tokens; base += stride) {
    int64_t my_next = -1;
#pragma unroll
    for (int r0 = 0; r0 < kGatherBatch; r0 += kGatherRows) {
      int64_t so[kGatherRows];
#pragma unroll
      for (int r = 0; r < kGatherRows; ++r) so[r] = __shfl_sync(0xffffffffu, my, r0 + r);
      for (int cb = 0; cb < nchunk; cb += 32 * kGatherSlots) {
        uint4 v[kGatherRows][kGatherSlots];
#pragma unroll
        for (int r = 0; r < kGatherRows; ++r)
#pragma unroll
          for (int k = 0; k < kGatherSlots; ++k) {
            const int c = cb + 32 * k + lane;
            v[r][k] = make_uint4(0u, 0u, 0u, 0u);
            if (so[r] >= 0 && c < nchunk) v[r][k] = ld_stream16(a.src + so[r] + 16 * (int64_t)c);
          }
        if (r0 == 0 && cb == 0 && base + stride < a.num_tokens) my_next = resolve(base + stride);
#pragma unroll
        for (int r = 0; r < kGatherRows; ++r) {
          uint8_t* drow = a.dst + (base + r0 + r) * a.dst_sr;
#pragma unroll
          for (int k = 0; k < kGatherSlots; ++k) {
            const int c = cb + 32 * k + lane;
            if (so[r] < 0 || c >= nchunk) continue;
            if (fp8) {
              float f[16];
              e4m3x16(v[r][k], sc, f);
              store16_vec(drow + (int64_t)c * 16 * dsz, a.dst_dt, f);
            } else if (same) {
              st_stream16(drow + 16 * (int64_t)c, v[r][k]);
            } else {
              const uint32_t w[4] = {v[r][k].x, v[r][k].y, v[r][k].z, v[r][k].w};
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const unsigned short e = (unsigned short)(w[q >> 1] >> (16 * (q & 1)));
                const float x = a.src_dt == QMLA_DT_BF16 ? __bfloat162float(__ushort_as_bfloat16(e))
                                                         : __half2float(__ushort_as_half(e));
                store_from_float(drow + ((int64_t)c * 8 + q) * dsz, a.dst_dt, x);
              }
            }
          }
        }
      }
      if (r0 == 0 && nchunk == 0 && base + stride < a.num_tokens) my_next = resolve(base + stride);
      // the columns the 16-byte chunks do not cover, and the FP8 rms tail
#pragma unroll 1
      for (int r = 0; r < kGatherRows; ++r) {
        const int64_t off = __shfl_sync(0xffffffffu, my, r0 + r);
        if (off < 0) continue;
        const uint8_t* srow = a.src + off;
        uint8_t* drow = a.dst + (base + r0 + r) * a.dst_sr;
        for (int c = nchunk * unit + lane; c < ncols; c += 32) {
          const float x = fp8 ? __fmul_rn(e4m3_to_float(srow[c]), sc) : load_as_float(srow + 2 * c, a.src_dt);
          store_from_float(drow + (int64_t)c * dsz, a.dst_dt, x);
        }
        for (int h = lane; h < a.rms_heads; h += 32) {
          float x;
          if (a.rms_mode == QMLA_RMS_LOG8) {
            // 2^(LO + code * (HI - LO) / 255), LO, HI = -3, 3, each step rounded to f32
            x = exp2f(__fadd_rn(-3.0f, __fmul_rn((float)srow[a.rms_off + h], 6.0f / 255.0f)));
          } else {
            const uint16_t bits = (uint16_t)srow[a.rms_off + 2 * h] |
                                  ((uint16_t)srow[a.rms_off + 2 * h + 1] << 8);
            x = __bfloat162float(__ushort_as_bfloat16(bits));
          }
          store_from_float(drow + (int64_t)(a.rms_off + h) * dsz, a.dst_dt, x);
        }
      }
    }
    my = my_next;
  }
}

// ---- staged variant: whole source rows through shared memory by the bulk-copy engine.
// Warp 8 (producer) resolves one stage's 32 row indices (one lane per row) and issues one
// cp.async.bulk per row into a ring of `stages` stages; warps 0-7 (converters) turn each
// staged row into the destination row.  The bytes in flight no longer depend on registers:
// stages - 1 stages per block are loading while one is converted.  Used when every row
// start is 16-byte aligned; the bytes of a row past its last whole 16-byte unit (and of any
// row longer than one stage slot) are read from global memory by the converters.
constexpr int kBulkConvWarps = 8;
constexpr int kBulkThreads = 32 * (kBulkConvWarps + 1);

struct BulkShape {
  int stages;      // ring depth, 2..8
  int rows;        // rows per stage (multiple of 8, <= 32)
  int slot;        // bytes per staged row (multiple of 16)
  int copy_bytes;  // bytes bulk-copied per row (multiple of 16, <= slot)
};

__host__ __device__ inline int bulk_smem_bytes(const BulkShape& b) {
  return b.stages * b.rows * b.slot + b.stages * b.rows * 8 + 2 * b.stages * 8 + 16;
}

__global__ void __launch_bounds__(kBulkThreads) gather_bulk_kernel(const GatherArgs a,
                                                                   const BulkShape sh) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = sh.stages;
  uint8_t* stage_buf = smem;
  int64_t* row_off = reinterpret_cast<int64_t*>(smem + S * sh.rows * sh.slot);
  uint64_t* bars = reinterpret_cast<uint64_t*>(row_off + S * sh.rows);  // full[S], empty[S]
  volatile int* abort_s = reinterpret_cast<volatile int*>(bars + 2 * S);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kBulkConvWarps);
    }
    *abort_s = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t nbatch = (a.num_tokens + sh.rows - 1) / sh.rows;
  if (warp == kBulkConvWarps) {
    // ---- producer
    const uint64_t pol = policy_evict_first();
    int i = 0;
    for (int64_t batch = blockIdx.x; batch < nbatch; batch += gridDim.x, ++i) {
      const int st = i % S;
      if (i >= S &&
          !mbar_wait(empty0 + 8 * st, (uint32_t)((i / S - 1) & 1), abort_s, a.status))
        break;
      const int64_t row = batch * sh.rows + lane;
      int64_t off = -1;
      if (lane < sh.rows && row < a.num_tokens) {
        off = gather_row_offset(a, row);
        if (off < 0 && a.status) atomicOr(a.status, QMLA_DEV_ERR_INDEX);
      }
      if (lane < sh.rows) row_off[st * sh.rows + lane] = off;
      const uint32_t mine = off >= 0 ? (uint32_t)sh.copy_bytes : 0u;
      const uint32_t total = __reduce_add_sync(0xffffffffu, mine);
      __syncwarp();
      if (lane == 0) mbar_expect_tx(full0 + 8 * st, total);  // the arrive publishes row_off
      __syncwarp();
      if (mine)
        bulk_load_1d(smem_u32(stage_buf + (st * sh.rows + lane) * sh.slot), a.src + off, mine,
                     full0 + 8 * st, pol);
    }
    // wait (bounded) until the copies of the last uses of every stage have landed, so that
    // none is in flight when the block exits
    const int issued = i;
    for (int u = issued - 1; u >= 0 && u >= issued - S; --u) {
      const int st = u % S;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(full0 + 8 * st, (uint32_t)((u / S) & 1)) &&
             globaltimer_ns() - t0 < 2000000000ull) {
      }
    }
    return;
  }
  // ---- converters: warp w takes rows w, w + 8, ... of each stage
  const int dsz = a.dst_dt == QMLA_DT_F32 ? 4 : 2;
  const float sc = a.scale ? __ldg(a.scale) : 1.0f;
  const bool fp8 = a.src_dt == QMLA_DT_FP8E4M3;
  const bool same = a.dst_dt == a.src_dt;
  const int unit = fp8 ? 16 : 8;
  const int ncols = fp8 ? a.n_e4m3 : a.n_copy;
  const int nchunk = min(ncols / unit, sh.copy_bytes / 16);  // chunks wholly inside the staged bytes
  int i = 0;
  for (int64_t batch = blockIdx.x; batch < nbatch; batch += gridDim.x, ++i) {
    const int st = i % S;
    if (!mbar_wait(full0 + 8 * st, (uint32_t)((i / S) & 1), abort_s, a.status)) break;
    for (int r = warp; r < sh.rows; r += kBulkConvWarps) {
      const int64_t off = row_off[st * sh.rows + r];
      if (off < 0) continue;
      const uint8_t* ss = stage_buf + (st * sh.rows + r) * sh.slot;
      const uint8_t* sg = a.src + off;
      uint8_t* drow = a.dst + (batch * sh.rows + r) * a.dst_sr;
      for (int c = lane; c < nchunk; c += 32) {
        const uint4 v = *reinterpret_cast<const uint4*>(ss + 16 * c);
        if (fp8) {
          float f[16];
          e4m3x16(v, sc, f);
          store16_vec(drow + (int64_t)c * 16 * dsz, a.dst_dt, f);
        } else if (same) {
          st_stream16(drow + 16 * (int64_t)c, v);
        } else {
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const unsigned short e = (unsigned short)(w[q >> 1] >> (16 * (q & 1)));
            const float x = a.src_dt == QMLA_DT_BF16 ? __bfloat162float(__ushort_as_bfloat16(e))
                                                     : __half2float(__ushort_as_half(e));
            store_from_float(drow + ((int64_t)c * 8 + q) * dsz, a.dst_dt, x);
          }
        }
      }
      auto byte_at = [&](int b) -> uint8_t { return b < sh.copy_bytes ? ss[b] : sg[b]; };
      for (int c = nchunk * unit + lane; c < ncols; c += 32) {
        float x;
        if (fp8) {
          x = __fmul_rn(e4m3_to_float(byte_at(c)), sc);
        } else {
          const unsigned short e = (unsigned short)(byte_at(2 * c) | (byte_at(2 * c + 1) << 8));
          x = a.src_dt == QMLA_DT_BF16 ? __bfloat162float(__ushort_as_bfloat16(e))
                                       : __half2float(__ushort_as_half(e));
        }
        store_from_float(drow + (int64_t)c * dsz, a.dst_dt, x);
      }
      for (int h = lane; h < a.rms_heads; h += 32) {
        float x;
        if (a.rms_mode == QMLA_RMS_LOG8) {
          x = exp2f(__fadd_rn(-3.0f, __fmul_rn((float)byte_at(a.rms_off + h), 6.0f / 255.0f)));
        } else {
          const uint16_t bits = (uint16_t)byte_at(a.rms_off + 2 * h) |
                                ((uint16_t)byte_at(a.rms_off + 2 * h + 1) << 8);
          x = __bfloat162float(__ushort_as_bfloat16(bits));
        }
        store_from_float(drow + (int64_t)(a.rms_off + h) * dsz, a.dst_dt, x);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * st);
  }
}

}  // namespace qmla
