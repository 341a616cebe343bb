// Decode-context-parallel merge over NVLink peer memory (sm_100a).
//
// Every rank of a DCP group owns one exchange buffer (ExchangeLayout below) that
// the other ranks have mapped through CUDA IPC.  A decode step writes the rank's
// partial (o, lse) for its KV shard into slot (epoch & 1) of its own buffer; the
// merge kernel then
//   1. publishes "epoch ready" into each peer's flag word for this rank (block 0 stores it; the
//      grid is at most a few blocks per SM, so every block is resident at once),
//   2. waits, bounded, until its own flag words show every peer at this epoch,
//   3. reads the N partials of its (row, head) items straight from the peers'
//      buffers and writes o = sum_n exp(lse_n - lse_g) o_n, lse_g = logsumexp lse_n
//      (NaN / +inf partial LSEs count as -inf, as in dcp_fix.py:62-98).
// Mode 1 gives rank r the heads [r*H/N, (r+1)*H/N) of every row (the layout of
// vLLM's cp_lse_ag_out_rs, which qwen_mla/dcp_fix.py:133-142 patches); mode 0
// gives every rank all heads.  One kernel replaces all-gather + correction +
// reduce-scatter.  Two slots let step e+1's decode write while peers may still
// read step e: a rank reaches step e+2's decode (slot e&1 again) only after its
// merge e+1 saw every peer's epoch-(e+1) flag, which a peer stores only once its
// merge e has finished reading.
#pragma once
#include <cuda_runtime.h>

#include "qmla_decode.cuh"

namespace qmla {

constexpr int kDcpMaxWorld = 8;
constexpr int kDcpHeader = 256;  // flags[kDcpMaxWorld] (u32), status (u32), padding, stats
constexpr int kDcpStatusOffset = 32;  // u32 status word (QMLA_DEV_ERR_* bits)
constexpr int kDcpEpochOffset = 36;   // u32 last epoch this rank merged (device-epoch mode)
constexpr int kDcpDoneOffset = 40;    // u32 blocks of the running merge that have finished
constexpr int kDcpStatsOffset = 64;   // u64 [launches, flag-wait ns, total ns, publish ns] of block 0

// Byte offsets inside one rank's exchange buffer.
struct ExchangeLayout {
  int64_t o_slot, lse_off, lse_slot, total;
  __host__ __device__ static ExchangeLayout make(int B, int H, int D) {
    ExchangeLayout L;
    L.o_slot = (((int64_t)B * H * D * 4) + 255) / 256 * 256;
    L.lse_off = kDcpHeader + 2 * L.o_slot;
    L.lse_slot = (((int64_t)B * H * 4) + 255) / 256 * 256;
    L.total = L.lse_off + 2 * L.lse_slot;
    return L;
  }
};

struct P2PArgs {
  uint8_t* bufs[kDcpMaxWorld];  // every rank's exchange buffer, mapped on this device
  int world, rank, B, H, D, mode;
  uint32_t epoch;  // 0: device-epoch mode (the epoch is the header's last epoch + 1)
  uint8_t* out;
  int64_t out_sr, out_sh;
  int out_dtype;
  float* lse_out;  // [B][H or H/world], natural log; may be null
  int64_t timeout_ns;
};

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// grid: up to a few blocks per SM, 128 threads; items = B x (heads of this rank).
__global__ void __launch_bounds__(128) dcp_p2p_merge_kernel(const P2PArgs a) {
  __shared__ float w_s[kDcpMaxWorld];
  __shared__ float lse_s;
  __shared__ int fail_s;
  const int tid = threadIdx.x;
  const ExchangeLayout L = ExchangeLayout::make(a.B, a.H, a.D);
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(a.bufs[a.rank]);
  // Block 0 stamps its entry, the end of its flag wait and its exit (%globaltimer) and adds the
  // wait and the total to the stats of this rank's own header: the host reads how long a step
  // waited for the slowest peer apart from the merge itself.
  const bool stamp = blockIdx.x == 0 && tid == 0;
  const uint64_t t_enter = stamp ? globaltimer_ns() : 0ull;
  // The step's epoch: the host's, or (epoch 0) one past the last epoch this rank merged, kept in
  // its own header so a replayed CUDA graph advances it.  The previous merge on this stream set
  // that word after all of its blocks had finished, so every block reads the same value.
  uint32_t* my_epoch = reinterpret_cast<uint32_t*>(a.bufs[a.rank] + kDcpEpochOffset);
  const uint32_t epoch = a.epoch != 0u ? a.epoch : *reinterpret_cast<volatile uint32_t*>(my_epoch) + 1u;
  // 1. publish: this rank's partial (written by the preceding decode on this stream, complete at
  // that kernel's end) is ready; one release store per peer, from block 0 only (a fence and a
  // remote store from every block of the grid cost microseconds per step)
  if (blockIdx.x == 0 && tid < a.world && tid != a.rank) {
    __threadfence_system();
    st_release_sys_u32(reinterpret_cast<uint32_t*>(a.bufs[tid]) + a.rank, epoch);
  }
  const uint64_t t_pub = stamp ? globaltimer_ns() : 0ull;
  // 2. wait (bounded) for every peer's flag in this rank's own buffer
  if (tid == 0) fail_s = 0;
  __syncthreads();
  if (tid < a.world && tid != a.rank) {
    const uint64_t t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys_u32(my_flags + tid) - epoch) < 0) {
      if (globaltimer_ns() - t0 > (uint64_t)a.timeout_ns) {
        fail_s = 1;
        atomicOr(reinterpret_cast<int*>(a.bufs[a.rank] + kDcpStatusOffset), QMLA_DEV_ERR_TIMEOUT);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  const uint64_t t_waited = stamp ? globaltimer_ns() : 0ull;
  // 3. merge (skipped after a wait that gave up; the epoch bookkeeping below still runs, so the
  // next step does not reuse this one's epoch)
  const int hs = a.mode == 1 ? a.H / a.world : a.H;
  const int h0 = a.mode == 1 ? a.rank * hs : 0;
  const int slot = (int)(epoch & 1u);
  const int n_items = fail_s ? 0 : a.B * hs;
  const int osz = dt_size(a.out_dtype);
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int b = item / hs, hl = item - b * hs, h = h0 + hl;
    if (tid < 32) {
      float v = -INFINITY;
      if (tid < a.world) {
        const float* lp = reinterpret_cast<const float*>(a.bufs[tid] + L.lse_off + slot * L.lse_slot);
        v = lp[(int64_t)b * a.H + h];
        if (v != v || v == INFINITY) v = -INFINITY;
      }
      float m = v;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const float e = (m == -INFINITY) ? 0.f : expf(v - m);
      float s = e;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (tid < a.world) w_s[tid] = s > 0.f ? e / s : 0.f;
      if (tid == 0) lse_s = s > 0.f ? m + logf(s) : -INFINITY;
    }
    __syncthreads();
    const int64_t obase = ((int64_t)b * a.H + h) * a.D;
    uint8_t* orow = a.out + ((int64_t)b * a.out_sr + (int64_t)hl * a.out_sh) * osz;
    for (int d4 = tid; d4 < a.D / 4; d4 += blockDim.x) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int n = 0; n < a.world; ++n) {
        const float w = w_s[n];
        if (w == 0.f) continue;
        const float4 v = *reinterpret_cast<const float4*>(
            a.bufs[n] + kDcpHeader + slot * L.o_slot + (obase + 4 * d4) * 4);
        acc.x += w * v.x;
        acc.y += w * v.y;
        acc.z += w * v.z;
        acc.w += w * v.w;
      }
      store_from_float(orow + (4 * d4 + 0) * osz, a.out_dtype, acc.x);
      store_from_float(orow + (4 * d4 + 1) * osz, a.out_dtype, acc.y);
      store_from_float(orow + (4 * d4 + 2) * osz, a.out_dtype, acc.z);
      store_from_float(orow + (4 * d4 + 3) * osz, a.out_dtype, acc.w);
    }
    if (tid == 0 && a.lse_out) a.lse_out[(int64_t)b * hs + hl] = lse_s;
    __syncthreads();  // w_s / lse_s are rewritten by the next item
  }
  // device-epoch mode: the last block to finish records this epoch as merged
  if (a.epoch == 0u && tid == 0) {
    unsigned int* done = reinterpret_cast<unsigned int*>(a.bufs[a.rank] + kDcpDoneOffset);
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      *reinterpret_cast<volatile uint32_t*>(my_epoch) = epoch;
      __threadfence();
    }
  }
  if (stamp) {
    unsigned long long* st = reinterpret_cast<unsigned long long*>(a.bufs[a.rank] + kDcpStatsOffset);
    atomicAdd(st + 0, 1ull);
    atomicAdd(st + 1, (unsigned long long)(t_waited - t_enter));
    atomicAdd(st + 2, (unsigned long long)(globaltimer_ns() - t_enter));
    atomicAdd(st + 3, (unsigned long long)(t_pub - t_enter));
  }
}

}  // namespace qmla
