// Persistent decode step of the Qwen3 forward: one cooperative launch runs a
// whole token (agent-test/v2/engine.py:145-163) instead of 143 kernels.
//
// Every CTA (128 threads, two per SM, all co-resident) walks the same phase
// sequence; a grid barrier separates phases whose inputs another CTA wrote:
//   embedding of the token
//   per layer:  norm + QKV GEMV | qk-norm + RoPE + KV append | split-KV decode
//               attention | O GEMV + residual | norm + gate/up GEMV + SwiGLU |
//               down GEMV + residual
//   final norm + LM-head GEMV with a fused argmax; the last CTA to finish
//   writes the next token and advances the position and key count.
// Rounding points are the model kernels' (model_kernels.cuh) and the units of
// the attention phase are decode_cta (decode_attention.cuh), so the results
// match the multi-kernel step up to FP32 summation order in the RMSNorm sums.
// Weight rows of the next GEMV phase are loaded into registers before each
// barrier, so each SM keeps streaming weights while the grid synchronises.
// Buffers written inside the kernel are read with L2-coherent loads (ld.cg);
// the K/V row written by the append phase reaches the attention phase's bulk
// copies through fence.proxy.async.global.
// Grid barrier: arrivals count on one word and the last arrival bumps a
// generation word that the others poll.  Every wait is bounded (common.cuh),
// and a CTA that gives up raises an abort flag that ends every other wait and
// phase.  Measured on B200 a barrier costs 3-4 us (one slot per CTA polled by
// every CTA costs 5 us): about as much as the kernel boundary it replaces, so
// this step is not faster than the CUDA graph of the multi-kernel step.
#pragma once

#include "common.cuh"
#include "decode_attention.cuh"
#include "model_kernels.cuh"
#include "qk_norm_rope.cuh"

namespace rib {
namespace step {

constexpr int kMaxLayers = 64;
constexpr int kMaxCtas = 1024;  // largest grid the launcher accepts
constexpr int NT = decode::NTHREADS;  // 128: the decode unit's CTA shape
constexpr int NWARP = NT / 32;

struct Layer {
  const uint16_t *qkv, *o, *gu, *down, *in_norm, *post_norm, *q_norm, *k_norm;
};

// Grid synchronisation words, in the workspace (zero before first use).
struct Sync {
  unsigned count;               // CTAs arrived at the current barrier
  unsigned gen;                 // barrier generation
  int abort;                    // a wait ran out: every CTA stops
  unsigned amax_done;           // CTAs done with the LM head
  unsigned long long amax_key;  // (value, -index) of the largest logit so far
};

struct Params {
  int L, hidden, nq, nkv, inter, vocab, cap;
  const uint16_t *embed, *final_norm;
  Layer layer[kMaxLayers];
  float inv_freq[64];   // rope_inv_freq
  const uint64_t *cache_ptrs;  // [L] layer caches [2][nkv][cap][128]
  int32_t *tok, *pos, *nkeys;  // device state: token in/out, position, key count
  uint16_t *h[3], *qkv, *q, *o, *a;
  float *logits;               // [vocab] FP32 or null
  Sync *sync;
  decode::Params dp;           // attention geometry and scratch (cache_ptrs set per layer)
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *a) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(unsigned *a, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int *a) { return *reinterpret_cast<const volatile int *>(a); }

// All CTAs of the grid.  False once any CTA has given up.
__device__ __forceinline__ bool grid_sync(Sync *sy, int *ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = !ld_volatile(&sy->abort);
    if (ok) {
      const unsigned gen = ld_acquire_gpu(&sy->gen);  // before arriving: the bump needs our arrival
      __threadfence();
      if (atomicAdd(&sy->count, 1u) == gridDim.x - 1) {
        atomicExch(&sy->count, 0u);
        __threadfence();
        st_release_gpu(&sy->gen, gen + 1);
      } else {
        const uint64_t t0 = global_timer_ns();
        while (ld_acquire_gpu(&sy->gen) == gen) {
          if (ld_volatile(&sy->abort)) {
            ok = 0;
            break;
          }
          if (global_timer_ns() - t0 > wait_limit_ns()) {
            record_timeout();
            atomicExch(&sy->abort, 1);
            ok = 0;
            break;
          }
        }
      }
      __threadfence();
    }
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

__device__ __forceinline__ void fail(Sync *sy, int status) {
  atomicExch(&g_device_status, status);
  atomicExch(&sy->abort, 1);
}

// x (BF16, written earlier in this kernel) into shared memory as FP32,
// RMSNorm'ed with weight nw when given (model_kernels.cuh rounding).
__device__ __forceinline__ void load_x(const uint16_t *x, const uint16_t *nw, int K, float *xs, float *red) {
  const int tid = threadIdx.x;
  float ss = 0.f;
  for (int i = tid * 8; i < K; i += NT * 8) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(x + i));
    const float f[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                        bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      xs[i + e] = f[e];
      ss = fmaf(f[e], f[e], ss);
    }
  }
  if (nw) {
    const float inv = 1.0f / sqrtf(model::block_sum(ss, red) / static_cast<float>(K) + model::kEps);
    for (int i = tid * 8; i < K; i += NT * 8) {
      const uint4 w = *reinterpret_cast<const uint4 *>(nw + i);
      const float wf[8] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y),
                           bf16lo(w.z), bf16hi(w.z), bf16lo(w.w), bf16hi(w.w)};
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[i + e] = round_bf16(wf[e] * round_bf16(xs[i + e] * inv));
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------ GEMV phases
// Warp gw of nw owns output rows gw, gw + nw, ...; the first MAXR of them are
// prefetched into registers (C = K / 256 chunks per lane known at compile
// time), the rest (small grids, or MAXR = 0) are streamed when computed.
template <int MAXR, int C, bool SW>
struct Pref {
  uint4 w[(SW ? 2 : 1) * (MAXR > 0 ? MAXR : 1)][C > 0 ? C : 1];
};

template <int MAXR, int C, bool SW>
__device__ __forceinline__ void gemv_prefetch(Pref<MAXR, C, SW> &pf, const uint16_t *W, int rows_out, int K,
                                              int gw, int nw, int lane) {
  if constexpr (MAXR > 0 && C > 0) {
#pragma unroll
    for (int i = 0; i < MAXR; ++i) {
      const int row = gw + i * nw;
      if (row < rows_out) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
          pf.w[i][c] = model::ldg_stream(W + static_cast<size_t>(row) * K + (c * 32 + lane) * 8);
          if constexpr (SW)
            pf.w[MAXR + i][c] =
                model::ldg_stream(W + static_cast<size_t>(row + rows_out) * K + (c * 32 + lane) * 8);
        }
      }
    }
  }
}

template <bool SW>
__device__ __forceinline__ void gemv_write(int row, float acc, float accu, int epi, const uint16_t *res,
                                           uint16_t *y) {
  float v;
  if (SW) {
    const float g = round_bf16(acc), u = round_bf16(accu);
    v = round_bf16(g * model::sigmoid_bf16(g)) * u;
  } else if (epi == model::kResidual) {
    const uint16_t r = __ldcg(reinterpret_cast<const unsigned short *>(res) + row);
    v = __uint_as_float(static_cast<uint32_t>(r) << 16) + round_bf16(acc);
  } else {
    v = acc;
  }
  y[row] = static_cast<uint16_t>(pack_bf16x2(v, 0.f) & 0xffffu);
}

template <int MAXR, int C, bool SW>
__device__ __forceinline__ void gemv_compute(const Pref<MAXR, C, SW> &pf, const uint16_t *W, int rows_out,
                                             int K, const float *xs, int epi, const uint16_t *res, uint16_t *y,
                                             int gw, int nw, int lane) {
  int first = gw;
  if constexpr (MAXR > 0 && C > 0) {
#pragma unroll
    for (int i = 0; i < MAXR; ++i) {
      const int row = gw + i * nw;
      if (row >= rows_out) break;
      float acc = 0.f, accu = 0.f;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const int col = (c * 32 + lane) * 8;
        const float4 xa = *reinterpret_cast<const float4 *>(xs + col);
        const float4 xb = *reinterpret_cast<const float4 *>(xs + col + 4);
        acc = model::dot8(pf.w[i][c], xa, xb, acc);
        if constexpr (SW) accu = model::dot8(pf.w[MAXR + i][c], xa, xb, accu);
      }
      acc = model::warp_sum(acc);
      if constexpr (SW) accu = model::warp_sum(accu);
      if (lane == 0) gemv_write<SW>(row, acc, accu, epi, res, y);
    }
    first = gw + MAXR * nw;
  }
  for (int row = first; row < rows_out; row += nw) {
    float acc = 0.f, accu = 0.f;
    for (int c = 0; c < K / 256; ++c) {
      const int col = (c * 32 + lane) * 8;
      const float4 xa = *reinterpret_cast<const float4 *>(xs + col);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + col + 4);
      acc = model::dot8(model::ldg_stream(W + static_cast<size_t>(row) * K + col), xa, xb, acc);
      if constexpr (SW)
        accu = model::dot8(model::ldg_stream(W + static_cast<size_t>(row + rows_out) * K + col), xa, xb, accu);
    }
    acc = model::warp_sum(acc);
    if constexpr (SW) accu = model::warp_sum(accu);
    if (lane == 0) gemv_write<SW>(row, acc, accu, epi, res, y);
  }
}

// LM head: logits = W_embed x (FP32), four rows per warp per pass, with the
// running argmax key of the rows this lane-0 wrote.
template <int C>
__device__ __forceinline__ unsigned long long lm_head(const Params &p, const float *xs, int gw, int nw,
                                                      int lane) {
  const int K = p.hidden;
  unsigned long long best = 0;
  for (int row0 = gw; row0 < p.vocab; row0 += 4 * nw) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int rows[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) rows[r] = min(row0 + r * nw, p.vocab - 1);
    const int nc = C > 0 ? C : K / 256;
#pragma unroll(C > 0 ? C : 1)
    for (int c = 0; c < nc; ++c) {
      const int col = (c * 32 + lane) * 8;
      uint4 w[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) w[r] = model::ldg_stream(p.embed + static_cast<size_t>(rows[r]) * K + col);
      const float4 xa = *reinterpret_cast<const float4 *>(xs + col);
      const float4 xb = *reinterpret_cast<const float4 *>(xs + col + 4);
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] = model::dot8(w[r], xa, xb, acc[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float v = model::warp_sum(acc[r]);
      const int row = row0 + r * nw;
      if (lane == 0 && row < p.vocab) {
        if (p.logits) p.logits[row] = v;
        const unsigned long long k = model::argmax_key(v, row);
        best = k > best ? k : best;
      }
    }
  }
  return best;
}

template <int CH, int CQ, int CI, int MQ, int MO, int MG, int MD>
__global__ void __launch_bounds__(NT, 2) decode_step_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  decode::Smem &s = *reinterpret_cast<decode::Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  float *xs = reinterpret_cast<float *>(&s.k[0][0]);  // GEMV input, aliases the attention ring
  __shared__ float red[32];
  __shared__ float cos_t[64], sin_t[64];
  __shared__ int ok_s;
  __shared__ unsigned long long best_s[NWARP];
  __shared__ bool last_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gw = blockIdx.x * NWARP + warp, nw = gridDim.x * NWARP;
  Sync *sy = p.sync;
  const int qkv_rows = (p.nq + 2 * p.nkv) * 128;
  const int q_dim = p.nq * 128;
  const int pos = *p.pos;

  // ---- embedding of the token
  if (blockIdx.x == 0) {
    const int t = *p.tok;
    if (t < 0 || t >= p.vocab || pos < 0 || pos >= p.cap) {
      if (tid == 0) fail(sy, t < 0 || t >= p.vocab ? RIB_EINVAL : RIB_ECAPACITY);
    } else {
      for (int c = tid * 8; c < p.hidden; c += NT * 8)
        *reinterpret_cast<uint4 *>(p.h[0] + c) =
            *reinterpret_cast<const uint4 *>(p.embed + static_cast<size_t>(t) * p.hidden + c);
    }
  }
  Pref<MQ, CH, false> pq;
  gemv_prefetch(pq, p.layer[0].qkv, qkv_rows, p.hidden, gw, nw, lane);
  bool ok = grid_sync(sy, &ok_s);

  int cur = 0;
  for (int l = 0; ok && l < p.L; ++l) {
    const Layer &w = p.layer[l];
    uint16_t *hin = p.h[cur], *h1 = p.h[(cur + 1) % 3], *hout = p.h[(cur + 2) % 3];

    // ---- norm + QKV GEMV
    load_x(hin, w.in_norm, p.hidden, xs, red);
    gemv_compute(pq, w.qkv, qkv_rows, p.hidden, xs, model::kNone, nullptr, p.qkv, gw, nw, lane);
    if (!(ok = grid_sync(sy, &ok_s))) break;

    // ---- qk-norm + RoPE of q and k, K/V append at `pos` (a half-warp per head)
    {
      const int items = p.nq + 2 * p.nkv;
      if (blockIdx.x * NWARP * 2 < items) {
        rope::rope_angles(pos, p.inv_freq, cos_t, sin_t, tid);
        __syncthreads();
        const int item = blockIdx.x * NWARP * 2 + warp * 2 + (lane >> 4);
        const int j = lane & 15;
        const unsigned half_mask = 0xffffu << (lane & 16);
        if (item < items) {
          const uint4 raw = __ldcg(reinterpret_cast<const uint4 *>(p.qkv + item * 128 + 8 * j));
          uint16_t *cache = reinterpret_cast<uint16_t *>(p.cache_ptrs[l]);
          if (item >= p.nq + p.nkv) {
            const int hv = item - p.nq - p.nkv;
            *reinterpret_cast<uint4 *>(cache + ((static_cast<size_t>(p.nkv + hv) * p.cap) + pos) * 128 + 8 * j) = raw;
          } else {
            const uint4 o = rope::norm_rope8(raw, item < p.nq ? w.q_norm : w.k_norm, j, half_mask, cos_t, sin_t);
            uint16_t *dst = item < p.nq ? p.q + item * 128 + 8 * j
                                        : cache + ((static_cast<size_t>(item - p.nq) * p.cap) + pos) * 128 + 8 * j;
            *reinterpret_cast<uint4 *>(dst) = o;
          }
        }
        asm volatile("fence.proxy.async.global;" ::: "memory");  // the new K/V row is read by bulk copies
      }
    }
    if (!(ok = grid_sync(sy, &ok_s))) break;

    // ---- split-KV decode attention of layer l
    {
      fence_proxy_async_smem();  // xs (generic writes) shares the ring the bulk copies fill
      decode::Params dp = p.dp;
      dp.cache_ptrs = p.cache_ptrs + l;
      const int units = dp.max_splits * p.nkv;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        decode::decode_cta(dp, s, u % dp.max_splits, u / dp.max_splits, 0);
        __syncthreads();
      }
    }
    Pref<MO, CQ, false> po;
    gemv_prefetch(po, w.o, p.hidden, q_dim, gw, nw, lane);
    if (!(ok = grid_sync(sy, &ok_s))) break;

    // ---- O GEMV + residual
    load_x(p.o, nullptr, q_dim, xs, red);
    gemv_compute(po, w.o, p.hidden, q_dim, xs, model::kResidual, hin, h1, gw, nw, lane);
    Pref<MG, CH, true> pg;
    gemv_prefetch(pg, w.gu, p.inter, p.hidden, gw, nw, lane);
    if (!(ok = grid_sync(sy, &ok_s))) break;

    // ---- norm + gate/up GEMV + SwiGLU
    load_x(h1, w.post_norm, p.hidden, xs, red);
    gemv_compute(pg, w.gu, p.inter, p.hidden, xs, model::kSwiGLU, nullptr, p.a, gw, nw, lane);
    Pref<MD, CI, false> pd;
    gemv_prefetch(pd, w.down, p.hidden, p.inter, gw, nw, lane);
    if (!(ok = grid_sync(sy, &ok_s))) break;

    // ---- down GEMV + residual
    load_x(p.a, nullptr, p.inter, xs, red);
    gemv_compute(pd, w.down, p.hidden, p.inter, xs, model::kResidual, h1, hout, gw, nw, lane);
    if (l + 1 < p.L) gemv_prefetch(pq, p.layer[l + 1].qkv, qkv_rows, p.hidden, gw, nw, lane);
    if (!(ok = grid_sync(sy, &ok_s))) break;
    cur = (cur + 2) % 3;
  }

  // ---- final norm + LM head + argmax; the last CTA writes the token
  if (!ok) return;
  load_x(p.h[cur], p.final_norm, p.hidden, xs, red);
  const unsigned long long best = lm_head<CH>(p, xs, gw, nw, lane);
  if (lane == 0) best_s[warp] = best;
  __syncthreads();
  if (tid == 0) {
    unsigned long long b = best_s[0];
    for (int i = 1; i < NWARP; ++i) b = best_s[i] > b ? best_s[i] : b;
    atomicMax(&sy->amax_key, b);
    __threadfence();
    last_s = atomicAdd(&sy->amax_done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last_s && tid == 0) {
    __threadfence();
    const unsigned long long b = atomicAdd(&sy->amax_key, 0ull);
    *p.tok = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(b & 0xffffffffull));
    *p.pos = pos + 1;
    *p.nkeys = pos + 2;
    sy->amax_key = 0;   // ready for the next step
    sy->amax_done = 0;
  }
}

}  // namespace step
}  // namespace rib
