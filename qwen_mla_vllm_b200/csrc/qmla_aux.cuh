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
__global__ void __launch_bounds__(1024) plan_kernel(const int32_t* __restrict__ seq_lens, int n,
                                                    int32_t* __restrict__ prefix,
                                                    int* __restrict__ status, int G, int seg_cost,
                                                    int32_t* __restrict__ bounds) {
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
      int L = seq_lens[i];
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
                                                     int32_t* __restrict__ bounds) {
  if (threadIdx.x == 0 && status) *status = 0;
  for (int c = threadIdx.x; c <= G; c += blockDim.x)
    bounds[c] = range_bound(prefix, n, G, seg_cost, c);
}

// Merge of the per-CTA partial segments of rows that crossed a CTA boundary
// (the reference's stage 2, mla_decode_attention.py:1064-1137, over the
// decode kernel's partition).  One block per (row, head); rows inside one CTA
// range are final already.  Rows of length 0 get o = 0 and lse = -inf.
__global__ void __launch_bounds__(128) split_merge_kernel(const DecodeArgs a) {
  const int row = blockIdx.x, h = blockIdx.y;
  const int plo = __ldg(a.tile_prefix + row), phi = __ldg(a.tile_prefix + row + 1);
  const int total = __ldg(a.tile_prefix + a.num_rows);
  const int H = a.H, D = a.rank;
  const int osz = dt_size(a.o_dtype);
  uint8_t* orow = a.o + ((int64_t)row * a.o_sr + (int64_t)h * a.o_sh) * osz;
  if (phi == plo) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) store_from_float(orow + d * osz, a.o_dtype, 0.f);
    if (a.lse && threadIdx.x == 0)
      store_from_float(a.lse + ((int64_t)row * a.lse_sr + h) * dt_size(a.lse_dtype), a.lse_dtype,
                       -INFINITY);
    return;
  }
  (void)total;
  // CTA ranges that hold tiles of this row (the decode kernel's partition, range_bounds)
  __shared__ int bnd[kMaxCtas + 1];
  for (int c = threadIdx.x; c <= a.G; c += blockDim.x) bnd[c] = __ldg(a.range_bounds + c);
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
  __shared__ float lse_g;
  __shared__ int np_s;
  if (threadIdx.x == 0) {
    int np = 0;  // empty ranges between c0 and c1 wrote nothing
    for (int c = c0; c <= c1; ++c)
      if (bnd[c] < bnd[c + 1]) slots[np++] = (plo <= bnd[c]) ? 2 * c : 2 * c + 1;
    np_s = np;
  }
  __syncthreads();
  const int np = np_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int i = 0; i < np; ++i) m = fmaxf(m, a.part_lse[(int64_t)slots[i] * H + h]);
    float sum = 0.f;
    for (int i = 0; i < np; ++i) {
      const float w = (m == -INFINITY) ? 0.f : exp2f(a.part_lse[(int64_t)slots[i] * H + h] - m);
      wts[i] = w;
      sum += w;
    }
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    for (int i = 0; i < np; ++i) wts[i] *= inv;
    lse_g = (m + log2f(sum)) * kLn2;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < np; ++i) acc += wts[i] * a.part_o[((int64_t)slots[i] * H + h) * D + d];
    store_from_float(orow + d * osz, a.o_dtype, acc);
  }
  if (a.lse && threadIdx.x == 0)
    store_from_float(a.lse + ((int64_t)row * a.lse_sr + h) * dt_size(a.lse_dtype), a.lse_dtype, lse_g);
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

}  // namespace qmla
