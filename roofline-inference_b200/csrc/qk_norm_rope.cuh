// Fused per-head RMSNorm + RoPE with the KV-cache append folded in.
//
// Semantics follow the reference Metal kernels agent-test/v2/kernels.py:116-146
// (one token) and :169-204 (L tokens):
//   inv  = 1 / sqrt(mean(x^2) + 1e-6)                      (kernels.py:129-130)
//   n_d  = bf16( w_d * bf16( x_d * inv ) )                  (kernels.py:131-133)
//   non-traditional RoPE, pairs (d, d+64), d in [0, 64):    (kernels.py:136-143)
//     theta_d = float(pos) * exp2(-(d/64) * log2(base)), all in FP32
//     o_d    = n_d cos - n_{d+64} sin,  o_{d+64} = n_d sin + n_{d+64} cos
//   V heads are copied bit for bit                         (kernels.py:123-127)
// The angle is the reference's FP32 value: the FP32 product -(d/64)*log2(base)
// (kernels.py:137-138, log2(base) rounded to FP32 as the Python f-string
// literal makes it, kernels.py:152), its exp2 rounded to FP32 on the host, and
// the FP32 product with float(pos).  mx.fast.rope forms theta the same way.
// Differences from the Metal source, by design:
//   - cos/sin of that FP32 angle are evaluated to full accuracy (reduced to
//     [-pi, pi] in FP64, then sincosf) where the Metal code calls
//     fast::cos / fast::sin, whose error grows with |theta|;
//   - K and V are written straight into the cache rows (engine.py:42-48 fused).
//
// Layout of the work: one CTA per token; each warp owns two (token, head)
// items, one per half-warp; lane j of a half-warp owns dims [8j, 8j+8), moved
// as one 16-byte vector.  The RoPE partner of dim d < 64 lives in lane j ^ 8.
#pragma once

#include <cmath>

#include "common.cuh"

namespace rib {
namespace rope {

constexpr int D = 128;
constexpr int kMaxItems = 64;  // nq + 2*nkv per token

struct Params {
  const uint16_t *qkv;  // [L][items*128]
  const uint16_t *qw;   // [128]
  const uint16_t *kw;   // [128]
  uint16_t *q_out;      // [nq][Lp][128]
  uint16_t *kv;         // [2][nkv][kv_rows][128]
  int L, Lp, offset, nq, nkv;
  int kv_rows;          // rows per head in kv (L, or the cache capacity)
  int kv_row0;          // first row written (0, or the cache offset)
  const int32_t *offset_dev;  // when set: the offset read on the device
  int rows_follow_offset;     // with offset_dev: K/V rows start at the device offset (cache
                              // append) rather than at kv_row0
  float inv_freq[64];   // exp2(-(d/64) log2(base)) rounded to FP32 (rope_inv_freq)
};

// Host: the 64 inverse frequencies exp2(-(d/64) * log2(base)) as the
// reference's FP32 arithmetic forms them (kernels.py:137-138, 152): log2(base)
// rounded to FP32, the FP32 product with -(d/64), and exp2 of that product
// rounded once to FP32.
inline void rope_inv_freq(float *out, double base) {
  const float lb = static_cast<float>(std::log2(base));
  for (int d = 0; d < 64; ++d) {
    volatile float x = -(static_cast<float>(d) / 64.0f) * lb;  // one FP32 rounding
    out[d] = static_cast<float>(std::exp2(static_cast<double>(x)));
  }
}

// cos/sin of the 64 RoPE angles at position `pos`: theta_d = float(pos) *
// inv_freq[d] as one FP32 product (kernels.py:134-138), then reduced to
// [-pi, pi] in FP64 and evaluated with the full-range sincosf.  Threads 0..63
// write.
__device__ __forceinline__ void rope_angles(int pos, const float *inv_freq, float *cos_t, float *sin_t,
                                            int tid) {
  if (tid < 64) {
    const double two_pi = 6.283185307179586476925286766559;
    const double th = static_cast<double>(__fmul_rn(static_cast<float>(pos), inv_freq[tid]));
    const double r = th - rint(th * (1.0 / two_pi)) * two_pi;
    float s, c;
    sincosf(static_cast<float>(r), &s, &c);
    cos_t[tid] = c;
    sin_t[tid] = s;
  }
}

// Per-head RMSNorm + RoPE of one head of 128 dims held by a half-warp: lane j
// (j = lane & 15) passes dims [8j, 8j+8) as `raw` and gets them back normed
// and rotated.  `w` is the head's norm weight (qw or kw).
__device__ __forceinline__ uint4 norm_rope8(const uint4 raw, const uint16_t *w, int j, unsigned half_mask,
                                            const float *cos_t, const float *sin_t) {
  float x[8];
  x[0] = bf16lo(raw.x); x[1] = bf16hi(raw.x);
  x[2] = bf16lo(raw.y); x[3] = bf16hi(raw.y);
  x[4] = bf16lo(raw.z); x[5] = bf16hi(raw.z);
  x[6] = bf16lo(raw.w); x[7] = bf16hi(raw.w);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(half_mask, ss, o, 16);
  const float inv = 1.0f / sqrtf(ss / 128.0f + 1e-6f);

  const uint4 wraw = *reinterpret_cast<const uint4 *>(w + 8 * j);
  float wf[8];
  wf[0] = bf16lo(wraw.x); wf[1] = bf16hi(wraw.x);
  wf[2] = bf16lo(wraw.y); wf[3] = bf16hi(wraw.y);
  wf[4] = bf16lo(wraw.z); wf[5] = bf16hi(wraw.z);
  wf[6] = bf16lo(wraw.w); wf[7] = bf16hi(wraw.w);

  float nv[8], pv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) nv[i] = round_bf16(wf[i] * round_bf16(x[i] * inv));
#pragma unroll
  for (int i = 0; i < 8; ++i) pv[i] = __shfl_xor_sync(half_mask, nv[i], 8, 16);

  const bool first_half = j < 8;
  const int a0 = 8 * (j & 7);
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float c = cos_t[a0 + i], s = sin_t[a0 + i];
    // first half: x1 = nv, x2 = pv ; second half: x1 = pv, x2 = nv
    o[i] = first_half ? fmaf(nv[i], c, -pv[i] * s) : fmaf(pv[i], s, nv[i] * c);
  }
  uint4 out;
  out.x = pack_bf16x2(o[0], o[1]);
  out.y = pack_bf16x2(o[2], o[3]);
  out.z = pack_bf16x2(o[4], o[5]);
  out.w = pack_bf16x2(o[6], o[7]);
  return out;
}

__global__ void __launch_bounds__(1024) qk_norm_rope_kernel(const __grid_constant__ Params p) {
  __shared__ float cos_t[64], sin_t[64];
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x;
  const int tid = threadIdx.x;
  int offset = p.offset, kv_row0 = p.kv_row0;
  if (p.offset_dev) {  // position kept on the device (CUDA-graph replay, no host sync)
    offset = *p.offset_dev;
    if (p.rows_follow_offset) kv_row0 = offset;
    if (offset < 0 || static_cast<long long>(kv_row0) + p.L > p.kv_rows) {
      if (t == 0 && tid == 0) atomicExch(&g_device_status, RIB_ECAPACITY);
      return;
    }
  }
  rope_angles(offset + t, p.inv_freq, cos_t, sin_t, tid);
  __syncthreads();

  const int items = p.nq + 2 * p.nkv;
  const int lane = tid & 31;
  const int item = (tid >> 5) * 2 + (lane >> 4);
  const int j = lane & 15;
  if (item >= items) return;
  const unsigned half_mask = 0xffffu << (lane & 16);

  if (t >= p.L) {  // padding rows of Q are zero (kernels.py:223, init_value=0)
    if (item < p.nq) {
      uint4 z = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4 *>(p.q_out + (static_cast<size_t>(item) * p.Lp + t) * D + 8 * j) = z;
    }
    return;
  }

  const uint4 raw = *reinterpret_cast<const uint4 *>(
      p.qkv + (static_cast<size_t>(t) * items + item) * D + 8 * j);

  if (item >= p.nq + p.nkv) {  // V: bit-exact copy into the cache
    const int hv = item - p.nq - p.nkv;
    uint16_t *dst = p.kv + ((static_cast<size_t>(p.nkv + hv) * p.kv_rows) + kv_row0 + t) * D + 8 * j;
    *reinterpret_cast<uint4 *>(dst) = raw;
    return;
  }

  const uint4 out = norm_rope8(raw, item < p.nq ? p.qw : p.kw, j, half_mask, cos_t, sin_t);
  uint16_t *dst;
  if (item < p.nq) {
    dst = p.q_out + (static_cast<size_t>(item) * p.Lp + t) * D + 8 * j;
  } else {
    const int hk = item - p.nq;
    dst = p.kv + ((static_cast<size_t>(hk) * p.kv_rows) + kv_row0 + t) * D + 8 * j;
  }
  *reinterpret_cast<uint4 *>(dst) = out;
}

}  // namespace rope
}  // namespace rib

namespace rib {
namespace rope {

// One new token for each of B sequences, each at its own position in its own
// cache: the batched form of the decode append (one CTA per sequence).
struct BatchParams {
  const uint16_t *qkv;          // [B][items*128]
  const uint16_t *qw, *kw;      // [128]
  uint16_t *q_out;              // [B][nq][128]
  const uint64_t *cache_ptrs;   // [B] caches [2][nkv][caps[b]][128]
  const int32_t *caps;          // [B]
  const int32_t *pos;           // [B] positions (the row written)
  int nq, nkv;
  float inv_freq[64];   // rope_inv_freq
};

__global__ void __launch_bounds__(1024) qk_norm_rope_batched_kernel(const __grid_constant__ BatchParams p) {
  __shared__ float cos_t[64], sin_t[64];
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x;
  const int pos = p.pos[b], cap = p.caps[b];
  if (pos < 0 || pos >= cap) {
    if (tid == 0) atomicExch(&g_device_status, RIB_ECAPACITY);
    return;
  }
  rope_angles(pos, p.inv_freq, cos_t, sin_t, tid);
  __syncthreads();
  const int items = p.nq + 2 * p.nkv;
  const int lane = tid & 31;
  const int item = (tid >> 5) * 2 + (lane >> 4);
  const int j = lane & 15;
  if (item >= items) return;
  const unsigned half_mask = 0xffffu << (lane & 16);
  const uint4 raw = *reinterpret_cast<const uint4 *>(p.qkv + (static_cast<size_t>(b) * items + item) * D + 8 * j);
  uint16_t *cache = reinterpret_cast<uint16_t *>(p.cache_ptrs[b]);
  if (item >= p.nq + p.nkv) {  // V: bit-exact copy
    const int hv = item - p.nq - p.nkv;
    *reinterpret_cast<uint4 *>(cache + (static_cast<size_t>(p.nkv + hv) * cap + pos) * D + 8 * j) = raw;
    return;
  }
  const uint4 out = norm_rope8(raw, item < p.nq ? p.qw : p.kw, j, half_mask, cos_t, sin_t);
  uint16_t *dst = item < p.nq ? p.q_out + (static_cast<size_t>(b) * p.nq + item) * D + 8 * j
                              : cache + (static_cast<size_t>(item - p.nq) * cap + pos) * D + 8 * j;
  *reinterpret_cast<uint4 *>(dst) = out;
}

}  // namespace rope
}  // namespace rib
