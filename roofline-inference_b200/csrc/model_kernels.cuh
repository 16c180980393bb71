// Kernels of the Qwen3 forward around the attention path: decode GEMVs with
// fused RMSNorm / residual / SwiGLU, the prefill residual+RMSNorm, RMSNorm,
// SwiGLU, the embedding gather and the greedy argmax.
//
// Rounding points follow the reference Metal kernels (agent-test/v2/kernels.py):
//   RMSNorm     inv = 1/sqrt(sum(x^2)/K + 1e-6), n = bf16(w * bf16(x * inv))
//               (kernels.py:48-55, 247-260)
//   GEMV        y = W x with FP32 accumulation, rounded once to BF16 (or kept
//               FP32 for the logits)                       (kernels.py:58-81)
//   residual    y = bf16(res + bf16(W x))                  (kernels.py:84-85)
//   SwiGLU      g = bf16(W_g x), u = bf16(W_u x), s = bf16(sigmoid(g)),
//               a = bf16(g s), y = bf16(a u)                (kernels.py:86-93)
//   add_rms     r = bf16(a + b), n = bf16(w * bf16(r * inv)) (kernels.py:227-268)
// The GEMVs are HBM-bound at batch 1: every weight byte is read once with
// 16-byte non-allocating loads, each warp owns R output rows and each lane
// covers K/256 16-byte chunks of a row, so one CTA of 8 warps keeps up to
// 8 * R * K * 2 bytes of weights in flight.  The input vector (normalised
// once per CTA when the RMSNorm is fused) sits in shared memory as FP32.
#pragma once

#include "common.cuh"

namespace rib {
namespace model {

constexpr float kEps = 1e-6f;
// Warps per GEMV CTA (a build-time tuning constant).
#ifndef RIB_GEMV_WARPS
#define RIB_GEMV_WARPS 8
#endif
constexpr int kGemvWarps = RIB_GEMV_WARPS;
// Warps per CTA of the wide form (RIB_GEMV_WIDE): half as many CTAs, each
// staging and normalising x once for twice the rows.  It pays after another
// GEMV; right after the decode attention the narrow CTAs fit beside the
// attention's and start their weight loads before it ends.
constexpr int kGemvWideWarps = 16;
constexpr int kMaxK = 8192;

enum Epilogue { kNone = 0, kResidual = 1, kSwiGLU = 2, kPeerPartial = 3 };

__device__ __forceinline__ void record_status(int status) { atomicExch(&g_device_status, status); }

// ------------------------------------------------------------------ tensor-parallel exchange
// rib_tp_exchange on the device.  Rank q's buffer holds [2 regions][world]
// [slot] 8-byte words; exchange e uses region e & 1, and rank r's values go
// to slot r.  Each word carries its value in the low 32 bits and the low 32
// bits of e in the high ones, written with one 8-byte store (single-copy
// atomic), so a reader that sees the epoch also sees the value: no fence, no
// separate flag and one NVLink crossing per exchange.  A region is rewritten
// two exchanges later, after every rank has read it (each rank produces
// exchange e + 1 only after consuming exchange e).
struct TpEx {
  int world, rank, slot;
  unsigned long long *buf[RIB_TP_MAX_RANKS];
  unsigned long long *epoch;  // this rank's exchange counter
  unsigned int *done;         // arrival counter of the producing kernel's warps
};

// Slot of `rank`'s words for exchange e, in rank q's buffer.
__device__ __forceinline__ unsigned long long *tp_slot(const TpEx &ex, int q, unsigned long long e, int rank) {
  return ex.buf[q] + (static_cast<size_t>(e & 1ull) * ex.world + rank) * ex.slot;
}

__device__ __forceinline__ unsigned long long tp_word(uint32_t value_bits, unsigned long long e) {
  return (static_cast<unsigned long long>(static_cast<uint32_t>(e)) << 32) | value_bits;
}

__device__ __forceinline__ void st_volatile_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ ulonglong2 ld_volatile_v2u64(const unsigned long long *p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}

// Two words of exchange e at p (16-byte aligned), polled until both carry
// e; gives up after wait_limit_ns() (shared deadline t0 per thread, 0: not
// started) with RIB_ETIMEOUT recorded.
__device__ __forceinline__ ulonglong2 tp_read2(const unsigned long long *p, unsigned long long e, uint64_t &t0) {
  const uint32_t want = static_cast<uint32_t>(e);
  ulonglong2 v = ld_volatile_v2u64(p);
  while (static_cast<uint32_t>(v.x >> 32) != want || static_cast<uint32_t>(v.y >> 32) != want) {
    const uint64_t now = global_timer_ns();
    if (t0 == 0) t0 = now;
    if (now - t0 > wait_limit_ns()) {
      record_timeout();
      break;
    }
    __nanosleep(32);
    v = ld_volatile_v2u64(p);
  }
  return v;
}

// 16-byte streaming load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the CTA (blockDim.x a multiple of 32, at most 1024); every thread
// gets the total.  `red` holds 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ float dot8(const uint4 w, const float4 xa, const float4 xb, float acc) {
  acc = fmaf(bf16lo(w.x), xa.x, acc);
  acc = fmaf(bf16hi(w.x), xa.y, acc);
  acc = fmaf(bf16lo(w.y), xa.z, acc);
  acc = fmaf(bf16hi(w.y), xa.w, acc);
  acc = fmaf(bf16lo(w.z), xb.x, acc);
  acc = fmaf(bf16hi(w.z), xb.y, acc);
  acc = fmaf(bf16lo(w.w), xb.z, acc);
  acc = fmaf(bf16hi(w.w), xb.w, acc);
  return acc;
}

// bf16(1 / (1 + exp(-g))) (agent-test/v2/kernels.py:89).  __fdividef is the
// branch-free approximate quotient (within 2 ulp of 1.0f / x for x below 2^126,
// 0 above, where the sigmoid is below 2^-126 anyway): the result is rounded to
// BF16 straight after, so it differs from the correctly rounded quotient's only
// when that lies within 2 FP32 ulp of a BF16 rounding boundary, and without the
// IEEE reciprocal's special-case branch the epilogues keep their elements in
// flight together.
__device__ __forceinline__ float sigmoid_bf16(float g) { return round_bf16(__fdividef(1.0f, 1.0f + expf(-g))); }

// ------------------------------------------------------------------ GEMV
struct GemvParams {
  const uint16_t *W;    // [N][K] BF16 row-major
  const uint16_t *x;    // [K]
  const uint16_t *nw;   // [K] RMSNorm weight, or null (no norm)
  const uint16_t *res;  // [rows_out] residual, epilogue kResidual
  void *y;              // [rows_out] BF16, or FP32 when out_f32
  int N, K, rows_out, epi, out_f32;
  // Tensor parallelism: with in_sum, x is the residual stream and the input
  // is bf16(x + bf16(sum of the last exchange's partials in rank order)),
  // written to x_out by CTA 0; epi kPeerPartial stores the FP32 rows into
  // every rank's exchange buffer and publishes the exchange.
  int in_sum;
  uint16_t *x_out;
  TpEx ex;
};

// C = K / 256 chunks of 8 elements per lane (0: runtime count); R output rows
// per warp; SW: SwiGLU epilogue (each output row reads its gate and up rows).
// The weight rows do not depend on the previous kernel, so with C known at
// compile time they are loaded into registers before the dependent-launch
// wait; x (and the residual) are read after it.
// TP: the tensor-parallel forms (in_sum input, kPeerPartial epilogue) are
// compiled in; without it those fields are ignored.
// W: warps per CTA (kGemvWarps, or kGemvWideWarps for the wide form).
template <int R, int C, bool SW, bool TP, int W = kGemvWarps>
__global__ void __launch_bounds__(W * 32) gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ float xs[];  // [K]
  __shared__ float red[32];
  pdl_launch_dependents();
  constexpr int NR = SW ? 2 * R : R;  // weight rows per warp
  const int K = p.K;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = (blockIdx.x * W + warp) * R;
  const bool active = row0 < p.rows_out;
  const int F = p.rows_out;  // up rows start at F in the SwiGLU case
  const uint16_t *wrow[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int rr = r < R ? min(row0 + r, p.rows_out - 1) : min(row0 + r - R, p.rows_out - 1) + F;
    wrow[r] = p.W + static_cast<size_t>(active ? rr : 0) * K;
  }
  uint4 wreg[NR][C > 0 ? C : 1];
  if (C > 0 && active) {
#pragma unroll
    for (int c = 0; c < (C > 0 ? C : 1); ++c)
#pragma unroll
      for (int r = 0; r < NR; ++r) wreg[r][c] = ldg_stream(wrow[r] + (c * 32 + lane) * 8);
  }
  // The norm weight is a model constant too: this thread's chunks of it (the
  // x chunks it stages below, at most kNwChunks of them) come in before the
  // wait as well.
  constexpr int kNwChunks = 2;
  const bool nw_pre = p.nw && K <= kNwChunks * static_cast<int>(W * 32) * 8;
  uint4 nwreg[kNwChunks];
  if (nw_pre) {
#pragma unroll
    for (int c = 0; c < kNwChunks; ++c) {
      const int i = (tid + c * W * 32) * 8;
      if (i < K) nwreg[c] = *reinterpret_cast<const uint4 *>(p.nw + i);
    }
  }
  pdl_wait();
  // The residual rows (written by an earlier kernel of the chain, complete
  // once the wait returns) are read now, so their latency overlaps x's.
  float resv[R];
  if (!SW && p.epi == kResidual && lane == 0 && active) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      resv[r] = row0 + r < p.rows_out ? __uint_as_float(static_cast<uint32_t>(p.res[row0 + r]) << 16) : 0.f;
  }

  // ---- x into shared memory (normalised when nw is given)
  const unsigned long long *part = nullptr;
  unsigned long long ex_e = 0;
  if (TP && p.in_sum) {
    ex_e = __ldcg(p.ex.epoch);  // the exchange the previous kernel published
    part = tp_slot(p.ex, p.ex.rank, ex_e, 0);
  }
  uint64_t t0 = 0;
  float ss = 0.f;
  auto stage8 = [&](int i, const uint4 v) {
    float f[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                  bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
    if (TP && part) {
      float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < p.ex.world; ++r) {
        const unsigned long long *src = part + static_cast<size_t>(r) * p.ex.slot + i;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const ulonglong2 w = tp_read2(src + 2 * j, ex_e, t0);
          sum[2 * j] += __uint_as_float(static_cast<uint32_t>(w.x));
          sum[2 * j + 1] += __uint_as_float(static_cast<uint32_t>(w.y));
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = round_bf16(f[e] + round_bf16(sum[e]));
      if (blockIdx.x == 0) {
        uint4 o;
        o.x = pack_bf16x2(f[0], f[1]);
        o.y = pack_bf16x2(f[2], f[3]);
        o.z = pack_bf16x2(f[4], f[5]);
        o.w = pack_bf16x2(f[6], f[7]);
        *reinterpret_cast<uint4 *>(p.x_out + i) = o;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      xs[i + e] = f[e];
      ss = fmaf(f[e], f[e], ss);
    }
  };
  for (int i = tid * 8; i < K; i += blockDim.x * 8) stage8(i, *reinterpret_cast<const uint4 *>(p.x + i));
  if (p.nw) {
    const float inv = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(K) + kEps);
    auto norm8 = [&](int i, const uint4 w) {
      const float wf[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                           bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[i + e] = round_bf16(wf[e] * round_bf16(xs[i + e] * inv));
    };
    if (nw_pre) {
#pragma unroll
      for (int c = 0; c < kNwChunks; ++c) {
        const int i = (tid + c * W * 32) * 8;
        if (i < K) norm8(i, nwreg[c]);
      }
    } else {
      for (int i = tid * 8; i < K; i += blockDim.x * 8) norm8(i, *reinterpret_cast<const uint4 *>(p.nw + i));
    }
  }
  __syncthreads();
  if (!active) return;

  float acc[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) acc[r] = 0.f;
  if (C > 0) {
#pragma unroll
    for (int c = 0; c < (C > 0 ? C : 1); ++c) {
      const int col = (c * 32 + lane) * 8;
      const float4 xa = *reinterpret_cast<const float4 *>(xs + col);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + col + 4);
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[r] = dot8(wreg[r][c], xa, xb, acc[r]);
    }
  } else {
    for (int c = 0; c < K / 256; ++c) {
      const int col = (c * 32 + lane) * 8;
      const float4 xa = *reinterpret_cast<const float4 *>(xs + col);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + col + 4);
      uint4 w[NR];
#pragma unroll
      for (int r = 0; r < NR; ++r) w[r] = ldg_stream(wrow[r] + col);
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[r] = dot8(w[r], xa, xb, acc[r]);
    }
    const int col = (K / 256) * 256 + lane * 8;  // K % 256 != 0: a partial chunk of K % 256 columns
    if (col < K) {
      const float4 xa = *reinterpret_cast<const float4 *>(xs + col);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + col + 4);
#pragma unroll
      for (int r = 0; r < NR; ++r) acc[r] = dot8(ldg_stream(wrow[r] + col), xa, xb, acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < NR; ++r) acc[r] = warp_sum(acc[r]);
  if (TP && !SW && p.epi == kPeerPartial) {
    // Lane q stores the warp's rows, tagged with the exchange's epoch, into
    // slot `rank` of rank q's buffer.  The last warp to finish (of
    // ceil(rows_out / R)) advances this rank's exchange counter.
    const unsigned long long e = __ldcg(p.ex.epoch) + 1;
    if (lane < p.ex.world) {
      unsigned long long *dst = tp_slot(p.ex, lane, e, p.ex.rank);
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (row0 + r < p.rows_out) st_volatile_u64(dst + row0 + r, tp_word(__float_as_uint(acc[r]), e));
    }
    if (lane == 0) {
      const unsigned int warps = static_cast<unsigned int>((p.rows_out + R - 1) / R);
      if (atomicAdd(p.ex.done, 1u) == warps - 1) {
        *p.ex.epoch = e;
        atomicExch(p.ex.done, 0u);
      }
    }
    return;
  }
  if (lane != 0) return;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    if (row >= p.rows_out) break;
    if (p.out_f32) {
      static_cast<float *>(p.y)[row] = acc[r];
      continue;
    }
    float v;
    if (SW) {
      const float g = round_bf16(acc[r]), u = round_bf16(acc[(SW ? R : 0) + r]);
      const float a = round_bf16(g * sigmoid_bf16(g));
      v = a * u;
    } else if (p.epi == kResidual) {
      v = resv[r] + round_bf16(acc[r]);
    } else {
      v = acc[r];
    }
    static_cast<uint16_t *>(p.y)[row] = static_cast<uint16_t>(pack_bf16x2(v, 0.f) & 0xffffu);
  }
}

// ------------------------------------------------------------------ row norms (prefill)
struct RowParams {
  const uint16_t *a;   // [rows][W]
  const uint16_t *b;   // [rows][W] added to a (add_rms), or null
  const uint16_t *w;   // [W] norm weight
  uint16_t *residual;  // [rows][W] a + b, or null
  uint16_t *out;       // [rows][W] normalised
  int rows, W;
};

// One warp per row for W = 256 * C: lane l holds the 16-byte chunks
// l, l + 32, ... of the row (8 elements each) in registers, the sum of
// squares is a warp reduction, and 8 rows share a CTA, so a long prompt runs
// a few hundred CTAs with every operand load issued up front.  Same rounding
// points as add_rms_kernel (the FP32 sum of squares adds in another order).
template <int C>
__global__ void __launch_bounds__(256) add_rms_rows_kernel(const __grid_constant__ RowParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const size_t base = static_cast<size_t>(row) * p.W;
  uint4 va[C], vb[C];
#pragma unroll
  for (int c = 0; c < C; ++c) va[c] = *reinterpret_cast<const uint4 *>(p.a + base + (c * 32 + lane) * 8);
  if (p.b) {
#pragma unroll
    for (int c = 0; c < C; ++c) vb[c] = *reinterpret_cast<const uint4 *>(p.b + base + (c * 32 + lane) * 8);
  }
  float f[C][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const uint4 a = va[c];
    f[c][0] = bf16lo(a.x); f[c][1] = bf16hi(a.x); f[c][2] = bf16lo(a.y); f[c][3] = bf16hi(a.y);
    f[c][4] = bf16lo(a.z); f[c][5] = bf16hi(a.z); f[c][6] = bf16lo(a.w); f[c][7] = bf16hi(a.w);
    if (p.b) {
      const uint4 b = vb[c];
      const float g[8] = {bf16lo(b.x), bf16hi(b.x), bf16lo(b.y), bf16hi(b.y),
                          bf16lo(b.z), bf16hi(b.z), bf16lo(b.w), bf16hi(b.w)};
#pragma unroll
      for (int e = 0; e < 8; ++e) f[c][e] = round_bf16(f[c][e] + g[e]);
      uint4 o;
      o.x = pack_bf16x2(f[c][0], f[c][1]);
      o.y = pack_bf16x2(f[c][2], f[c][3]);
      o.z = pack_bf16x2(f[c][4], f[c][5]);
      o.w = pack_bf16x2(f[c][6], f[c][7]);
      *reinterpret_cast<uint4 *>(p.residual + base + (c * 32 + lane) * 8) = o;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(f[c][e], f[c][e], ss);
  }
  const float inv = 1.0f / sqrtf(warp_sum(ss) / static_cast<float>(p.W) + kEps);
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

// One CTA per row, 8 elements per thread per step.  The row is kept in
// shared memory between the sum of squares and the normalisation.
__global__ void __launch_bounds__(256) add_rms_kernel(const __grid_constant__ RowParams p) {
  extern __shared__ float rs[];  // [W]
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const size_t base = static_cast<size_t>(blockIdx.x) * p.W;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < p.W; i += blockDim.x * 8) {
    const uint4 va = *reinterpret_cast<const uint4 *>(p.a + base + i);
    float f[8] = {bf16lo(va.x), bf16hi(va.x), bf16lo(va.y), bf16hi(va.y),
                  bf16lo(va.z), bf16hi(va.z), bf16lo(va.w), bf16hi(va.w)};
    if (p.b) {
      const uint4 vb = *reinterpret_cast<const uint4 *>(p.b + base + i);
      const float g[8] = {bf16lo(vb.x), bf16hi(vb.x), bf16lo(vb.y), bf16hi(vb.y),
                          bf16lo(vb.z), bf16hi(vb.z), bf16lo(vb.w), bf16hi(vb.w)};
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = round_bf16(f[e] + g[e]);
      uint4 o;
      o.x = pack_bf16x2(f[0], f[1]);
      o.y = pack_bf16x2(f[2], f[3]);
      o.z = pack_bf16x2(f[4], f[5]);
      o.w = pack_bf16x2(f[6], f[7]);
      *reinterpret_cast<uint4 *>(p.residual + base + i) = o;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      rs[i + e] = f[e];
      ss = fmaf(f[e], f[e], ss);
    }
  }
  const float inv = 1.0f / sqrtf(block_sum(ss, red) / static_cast<float>(p.W) + kEps);
  for (int i = threadIdx.x * 8; i < p.W; i += blockDim.x * 8) {
    const uint4 w = *reinterpret_cast<const uint4 *>(p.w + i);
    const float wf[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                         bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
    float n[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) n[e] = wf[e] * round_bf16(rs[i + e] * inv);
    uint4 o;
    o.x = pack_bf16x2(n[0], n[1]);
    o.y = pack_bf16x2(n[2], n[3]);
    o.z = pack_bf16x2(n[4], n[5]);
    o.w = pack_bf16x2(n[6], n[7]);
    *reinterpret_cast<uint4 *>(p.out + base + i) = o;
  }
}

// ------------------------------------------------------------------ SwiGLU (prefill)
// gu [rows][2F] (gate columns [0, F), up columns [F, 2F)) -> out [rows][F].
__global__ void swiglu_kernel(const uint16_t *__restrict__ gu, int rows, int F, uint16_t *__restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const long long total = static_cast<long long>(rows) * (F / 8);
  for (long long v = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < total;
       v += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = v / (F / 8);
    const int c = static_cast<int>(v - r * (F / 8)) * 8;
    const uint4 g4 = *reinterpret_cast<const uint4 *>(gu + r * 2 * F + c);
    const uint4 u4 = *reinterpret_cast<const uint4 *>(gu + r * 2 * F + F + c);
    const float g[8] = {bf16lo(g4.x), bf16hi(g4.x), bf16lo(g4.y), bf16hi(g4.y),
                        bf16lo(g4.z), bf16hi(g4.z), bf16lo(g4.w), bf16hi(g4.w)};
    const float u[8] = {bf16lo(u4.x), bf16hi(u4.x), bf16lo(u4.y), bf16hi(u4.y),
                        bf16lo(u4.z), bf16hi(u4.z), bf16lo(u4.w), bf16hi(u4.w)};
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = round_bf16(g[e] * sigmoid_bf16(g[e])) * u[e];
    uint4 o;
    o.x = pack_bf16x2(y[0], y[1]);
    o.y = pack_bf16x2(y[2], y[3]);
    o.z = pack_bf16x2(y[4], y[5]);
    o.w = pack_bf16x2(y[6], y[7]);
    *reinterpret_cast<uint4 *>(out + r * F + c) = o;
  }
}

// ------------------------------------------------------------------ embedding gather
// out[i] = table[tokens[i]]; a token outside [0, vocab) writes zeros and
// records RIB_EINVAL in the device status word.
__global__ void embed_kernel(const uint16_t *__restrict__ table, int vocab, int hidden,
                             const int32_t *__restrict__ tokens, uint16_t *__restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x;
  const int tok = tokens[i];
  const bool ok = tok >= 0 && tok < vocab;
  if (!ok && threadIdx.x == 0) record_status(RIB_EINVAL);
  for (int c = threadIdx.x * 8; c < hidden; c += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (ok) v = *reinterpret_cast<const uint4 *>(table + static_cast<size_t>(tok) * hidden + c);
    *reinterpret_cast<uint4 *>(out + static_cast<size_t>(i) * hidden + c) = v;
  }
}

// ------------------------------------------------------------------ greedy argmax
// Index of the largest FP32 value (the first one on ties, as numpy/MLX argmax).
// Keys order (value, -index) as unsigned 64-bit integers; each CTA folds its
// slice into ws->best with atomicMax, and the last CTA to finish (counted in
// ws->done) writes the index.  The caller clears the workspace first.
struct ArgmaxWs {
  unsigned long long best;
  unsigned int done;
};

__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // monotone in v
  return (static_cast<unsigned long long>(b) << 32) | (0xffffffffu - static_cast<uint32_t>(i));
}

__global__ void __launch_bounds__(1024) argmax_kernel(const float *__restrict__ x, int n, ArgmaxWs *ws,
                                                      int32_t *__restrict__ out) {
  __shared__ unsigned long long red[32];
  __shared__ bool last;
  pdl_launch_dependents();
  pdl_wait();
  unsigned long long best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = argmax_key(x[i], i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    atomicMax(&ws->best, best);
    __threadfence();
    last = atomicAdd(&ws->done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    const unsigned long long b = atomicAdd(&ws->best, 0ull);
    out[0] = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffull));
  }
}

// Greedy token over the ranks' logit slices (tensor-parallel LM head): x
// holds logits [offset, offset + n); keys carry the global index.  The last
// CTA publishes this rank's best key to every rank (one exchange), waits
// (bounded) for every rank's key and writes the largest key's index.
__global__ void __launch_bounds__(1024) argmax_tp_kernel(const float *__restrict__ x, int n, int offset,
                                                         ArgmaxWs *ws, int32_t *__restrict__ out,
                                                         const __grid_constant__ TpEx ex) {
  __shared__ unsigned long long red[32];
  __shared__ bool last;
  pdl_launch_dependents();
  pdl_wait();
  unsigned long long best = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const unsigned long long k = argmax_key(x[i], i + offset);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    atomicMax(&ws->best, best);
    __threadfence();
    last = atomicAdd(&ws->done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  const unsigned long long mine = atomicAdd(&ws->best, 0ull);
  const unsigned long long e = __ldcg(ex.epoch) + 1;
  // this rank's key as two tagged words (low, high half) in every rank's slot
  for (int q = 0; q < ex.world; ++q) {
    unsigned long long *dst = tp_slot(ex, q, e, ex.rank);
    st_volatile_u64(dst, tp_word(static_cast<uint32_t>(mine), e));
    st_volatile_u64(dst + 1, tp_word(static_cast<uint32_t>(mine >> 32), e));
  }
  unsigned long long g = 0;
  uint64_t t0 = 0;
  for (int r = 0; r < ex.world; ++r) {
    const ulonglong2 v = tp_read2(tp_slot(ex, ex.rank, e, r), e, t0);
    const unsigned long long k = (static_cast<unsigned long long>(static_cast<uint32_t>(v.y)) << 32) |
                                 static_cast<uint32_t>(v.x);
    g = k > g ? k : g;
  }
  out[0] = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(g & 0xffffffffull));
  *ex.epoch = e;
}

// Greedy token of each row of x [rows][n] (the first index on ties): one CTA
// of 1024 threads per row, the same keys as argmax_kernel.  The row body is
// read as 16-byte vectors, four per thread in flight (64 KB per CTA), with a
// scalar head up to the first 16-byte boundary and a scalar tail.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float *__restrict__ x, int n,
                                                           int32_t *__restrict__ out) {
  __shared__ unsigned long long red[32];
  pdl_launch_dependents();
  pdl_wait();
  const float *row = x + static_cast<size_t>(blockIdx.x) * n;
  const int t = threadIdx.x, nt = blockDim.x;
  unsigned long long best = 0;
  const int mis = static_cast<int>((reinterpret_cast<uintptr_t>(row) >> 2) & 3u);
  const int head = min(n, (4 - mis) & 3);
  if (t < head) best = argmax_key(__ldcs(row + t), t);
  const int nv = (n - head) >> 2;
  const float4 *v = reinterpret_cast<const float4 *>(row + head);
  for (int j = t; j < nv; j += 4 * nt) {
    float4 a[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (j + u * nt < nv) a[u] = __ldcs(v + j + u * nt);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int jj = j + u * nt;
      if (jj < nv) {
        const int i = head + 4 * jj;
        unsigned long long k = argmax_key(a[u].x, i);
        best = k > best ? k : best;
        k = argmax_key(a[u].y, i + 1);
        best = k > best ? k : best;
        k = argmax_key(a[u].z, i + 2);
        best = k > best ? k : best;
        k = argmax_key(a[u].w, i + 3);
        best = k > best ? k : best;
      }
    }
  }
  const int tail0 = head + 4 * nv;
  if (tail0 + t < n) {
    const unsigned long long k = argmax_key(__ldcs(row + tail0 + t), tail0 + t);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((t & 31) == 0) red[t >> 5] = best;
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < (nt >> 5); ++w) best = red[w] > best ? red[w] : best;
    out[blockIdx.x] = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(best & 0xffffffffull));
  }
}

}  // namespace model
}  // namespace rib
