// Tensor-parallel prefill: the exchange after a row-parallel projection
// (O, down), fused over NVLink peer memory.
//
// Under tensor parallelism each rank's O and down GEMMs produce FP32 partial
// sums [M][H] of the hidden state; the next step needs on every rank
// residual + bf16(sum of the ranks' partials), then the RMSNorm of that
// (agent-test/v2/kernels.py:227-268, the add_rms after each projection of
// Engine.prefill, agent-test/v2/engine.py:111-116).  Two kernels do it:
//
//   1. gemm_kernel with the kF32Owner epilogue: rows are owned by ranks in
//      contiguous runs of rpo = ceil(M / world); each tile row's FP32
//      partial is stored straight into its owner's receive slot for this
//      rank -- a reduce-scatter inside the GEMM, overlapping the next tile's
//      MMAs -- and each epilogue thread ends with a system-scope fence;
//   2. tp_reduce_add_rms_kernel below: signal "my partials are in place" to
//      every rank and wait for every rank's signal; sum the owned rows'
//      partials in rank order (deterministic), round to BF16 and store the
//      row into every rank's gather buffer (an all-gather of BF16 rows); the
//      CTA that completes the rank's rows signals "my rows are in place";
//      every CTA waits for every rank's rows and runs the residual add and
//      RMSNorm of all M rows with the rounding points of add_rms_rows_kernel.
//
// Per rank and exchange the GEMM sends (world - 1) / world of its partials
// (FP32) and the reduce kernel (world - 1) / world of the reduced rows (BF16)
// over NVLink, the traffic of a ring all-reduce, with no NCCL launch.
//
// Buffer reuse is ordered by the flags alone: a rank's next GEMM stores into
// an owner's receive slots only after that owner's "rows in place" signal,
// which the owner sends after it has read its slots; an owner stores into a
// rank's gather buffer only after that rank's next "partials in place"
// signal, sent after it has read the buffer.  Every wait is bounded
// (wait_limit_ns); on a timeout the kernel records RIB_ETIMEOUT and returns.
// Plain loads and stores over NVLink only; no TMA, no multicast.
#pragma once

#include "common.cuh"
#include "model_kernels.cuh"

namespace rib {
namespace tpp {

constexpr int kMaxRanks = 8;
// Threads per CTA for H = 256 C: 16 warps (one row per warp at a time) up to
// H = 1024, 8 at H = 2048, whose rows take twice the registers.
template <int C>
__host__ __device__ constexpr int threads_for() { return C <= 4 ? 512 : 256; }

// Layout of one rank's exchange buffer (bytes from its base):
//   [0, 128)          flags: u64 [2][8], [0][s] = source s's partials are in
//                     place, [1][s] = source s's reduced rows are in place
//   [128, 132)        the CTA counter of the reduce kernel (zero between launches)
//   [256, ...)        receive slots: FP32 [world][rpo_cap][H]
//   then              gather buffer: BF16 [rows_cap][H] (256-byte aligned)
constexpr size_t kFlagsOffset = 0;
constexpr size_t kCounterOffset = 128;
constexpr size_t kRecvOffset = 256;

__host__ __device__ inline int rows_per_owner(int rows, int world) { return (rows + world - 1) / world; }
__host__ __device__ inline size_t recv_bytes(int world, int rows_cap, int H) {
  return static_cast<size_t>(world) * rows_per_owner(rows_cap, world) * H * sizeof(float);
}
__host__ __device__ inline size_t gather_offset(int world, int rows_cap, int H) {
  return (kRecvOffset + recv_bytes(world, rows_cap, H) + 255) / 256 * 256;
}
__host__ __device__ inline size_t buffer_bytes(int world, int rows_cap, int H) {
  return gather_offset(world, rows_cap, H) + static_cast<size_t>(rows_cap) * H * 2;
}

struct ReduceParams {
  unsigned long long *flags[kMaxRanks];  // each rank's flag words, as seen from here
  uint16_t *gather[kMaxRanks];           // each rank's gather buffer [rows_cap][H]
  const float *recv;                     // this rank's receive slots [world][rpo_cap][H]
  int *counter;                          // this rank's CTA counter
  unsigned long long epoch;              // > every epoch used before on these buffers
  long long slot_floats;                 // rpo_cap * H
  int world, rank, M, H, rpo;
  uint16_t *residual;                    // [M][H]: in h, out bf16(h + r)
  const uint16_t *w;                     // [H] RMSNorm weight, or null (residual add only)
  uint16_t *out;                         // [M][H] normalised rows (when w)
};

// Bounded wait of one thread for *flag >= epoch; false on a timeout.
__device__ __forceinline__ bool wait_flag(const unsigned long long *flag, unsigned long long epoch) {
  if (ld_acquire_sys(flag) >= epoch) return true;
  const uint64_t t0 = global_timer_ns();
  while (ld_acquire_sys(flag) < epoch) {
    if (global_timer_ns() - t0 > wait_limit_ns()) {
      record_timeout();
      return false;
    }
  }
  return true;
}

// Threads [0, world) wait for flag word `which` of every source; the CTA
// learns whether all arrived.
__device__ __forceinline__ bool wait_all(const ReduceParams &p, int which, int *s_ok) {
  if (threadIdx.x == 0) *s_ok = 1;
  __syncthreads();
  if (threadIdx.x < p.world && !wait_flag(p.flags[p.rank] + which * kMaxRanks + threadIdx.x, p.epoch)) *s_ok = 0;
  __syncthreads();
  return *s_ok != 0;
}

template <int C>  // H = 256 C: lane l holds the 16-byte chunks l, l + 32, ... of a row
__global__ void __launch_bounds__(threads_for<C>()) tp_reduce_add_rms_kernel(const __grid_constant__ ReduceParams p) {
  constexpr int kWarps = threads_for<C>() / 32;
  __shared__ int s_ok, s_last;
  pdl_launch_dependents();
  pdl_wait();  // this rank's GEMM (and its fences) are complete
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;

  // ---- 1. partials in place everywhere
  if (blockIdx.x == 0 && threadIdx.x < p.world) {
    __threadfence_system();
    st_release_sys(p.flags[threadIdx.x] + p.rank, p.epoch);
  }
  if (!wait_all(p, 0, &s_ok)) return;

  // ---- 2. owned rows: sum of the partials in rank order, BF16, to every rank
  const int r0 = p.rank * p.rpo, r1 = min(p.M, r0 + p.rpo);
  for (int row = r0 + gw; row < r1; row += nw) {
    float acc[C][8];
    const size_t off = static_cast<size_t>(row - r0) * p.H;
#pragma unroll 1
    for (int s = 0; s < p.world; ++s) {
      const float4 *src = reinterpret_cast<const float4 *>(p.recv + s * p.slot_floats + off);
      float4 v[C][2];
#pragma unroll
      for (int c = 0; c < C; ++c) {
        v[c][0] = __ldcg(src + (c * 32 + lane) * 2);
        v[c][1] = __ldcg(src + (c * 32 + lane) * 2 + 1);
      }
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const float e[8] = {v[c][0].x, v[c][0].y, v[c][0].z, v[c][0].w, v[c][1].x, v[c][1].y, v[c][1].z, v[c][1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[c][i] = s == 0 ? e[i] : acc[c][i] + e[i];
      }
    }
    uint4 o[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      o[c].x = pack_bf16x2(acc[c][0], acc[c][1]);
      o[c].y = pack_bf16x2(acc[c][2], acc[c][3]);
      o[c].z = pack_bf16x2(acc[c][4], acc[c][5]);
      o[c].w = pack_bf16x2(acc[c][6], acc[c][7]);
    }
#pragma unroll 1
    for (int t = 0; t < p.world; ++t) {
      const int dst_rank = (p.rank + t) % p.world;  // start with this rank's own copy
      uint4 *dst = reinterpret_cast<uint4 *>(p.gather[dst_rank] + static_cast<size_t>(row) * p.H);
#pragma unroll
      for (int c = 0; c < C; ++c) dst[c * 32 + lane] = o[c];
    }
  }

  // ---- 3. the CTA that completes this rank's rows signals every rank
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    s_last = atomicAdd(p.counter, 1) == static_cast<int>(gridDim.x) - 1;
  }
  __syncthreads();
  if (s_last) {
    if (threadIdx.x == 0) {
      atomicExch(p.counter, 0);
      __threadfence_system();
    }
    __syncthreads();
    if (threadIdx.x < p.world) st_release_sys(p.flags[threadIdx.x] + kMaxRanks + p.rank, p.epoch);
  }
  if (!wait_all(p, 1, &s_ok)) return;

  // ---- 4. every row: residual add and RMSNorm (add_rms_rows_kernel's rounding)
  const uint16_t *g = p.gather[p.rank];
  for (int row = gw; row < p.M; row += nw) {
    const size_t base = static_cast<size_t>(row) * p.H;
    uint4 va[C], vb[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
      va[c] = *reinterpret_cast<const uint4 *>(p.residual + base + (c * 32 + lane) * 8);
      vb[c] = __ldcg(reinterpret_cast<const uint4 *>(g + base + (c * 32 + lane) * 8));
    }
    float f[C][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const uint4 a = va[c], b = vb[c];
      const float fa[8] = {bf16lo(a.x), bf16hi(a.x), bf16lo(a.y), bf16hi(a.y),
                           bf16lo(a.z), bf16hi(a.z), bf16lo(a.w), bf16hi(a.w)};
      const float fb[8] = {bf16lo(b.x), bf16hi(b.x), bf16lo(b.y), bf16hi(b.y),
                           bf16lo(b.z), bf16hi(b.z), bf16lo(b.w), bf16hi(b.w)};
#pragma unroll
      for (int e = 0; e < 8; ++e) f[c][e] = round_bf16(fa[e] + fb[e]);
      uint4 o;
      o.x = pack_bf16x2(f[c][0], f[c][1]);
      o.y = pack_bf16x2(f[c][2], f[c][3]);
      o.z = pack_bf16x2(f[c][4], f[c][5]);
      o.w = pack_bf16x2(f[c][6], f[c][7]);
      *reinterpret_cast<uint4 *>(p.residual + base + (c * 32 + lane) * 8) = o;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(f[c][e], f[c][e], ss);
    }
    if (!p.w) continue;
    const float inv = 1.0f / sqrtf(model::warp_sum(ss) / static_cast<float>(p.H) + model::kEps);
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const uint4 w = *reinterpret_cast<const uint4 *>(p.w + (c * 32 + lane) * 8);
      const float wf[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                           bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
      float n[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) n[e] = wf[e] * round_bf16(f[c][e] * inv);
      uint4 o;
      o.x = pack_bf16x2(n[0], n[1]);
      o.y = pack_bf16x2(n[2], n[3]);
      o.z = pack_bf16x2(n[4], n[5]);
      o.w = pack_bf16x2(n[6], n[7]);
      *reinterpret_cast<uint4 *>(p.out + base + (c * 32 + lane) * 8) = o;
    }
  }
}

}  // namespace tpp
}  // namespace rib
