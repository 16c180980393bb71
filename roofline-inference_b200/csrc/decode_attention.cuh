// GQA split-KV decode attention (flash-decoding) for sm_100a.
//
// Replaces the MLX library call mx.fast.scaled_dot_product_attention(q, K, V,
// scale) made by Engine.decode (agent-test/v2/engine.py:154-155): one query
// token per sequence, q heads 2h and 2h+1 read KV head h (GQA group 2), no
// mask, n = offset + 1 keys (engine.py:149).
//
// Work split: CTA (split, kv_head, seq) streams keys [split*chunk,
// min(n, (split+1)*chunk)) of one KV head for both of its query heads.
//   - warp NCW (producer): one lane issues 1-D bulk copies (cp.async.bulk) of
//     K and V tiles of TK keys into a STAGES-deep shared-memory ring; each
//     tile of one head is a contiguous TK*256-byte run of the cache, so no
//     tensor map is needed.  L2 policy evict_first: the cache is read once.
//   - warps 0-2 (consumers) take tiles round-robin (tile t -> warp t % NCW)
//     and each warp owns SPW ring slots of its own, so a warp waits on the
//     next phase of a slot only after it consumed the previous one itself
//     (a slot shared between warps could be waited on one phase early, and
//     an mbarrier parity wait cannot tell phase k from phase k + 2).
//     Scores: an 8-lane group
//     owns 8 keys, lane j of the group holds dims [8j,8j+8) and [64+8j,64+8j+8)
//     (two 16-byte conflict-free shared loads per key), a 3-step butterfly
//     reduce-scatter leaves lane l with the full score of key l for both
//     heads.  Online softmax in the exp2 domain (q pre-scaled by
//     scale*log2 e), warp-uniform running max.  P.V: lane l owns dims
//     [4l, 4l+4) and accumulates all keys of the tile for both heads in FP32.
//   - The CTA merges its consumer warps in shared memory.  With one split the CTA
//     writes the BF16 output; otherwise it writes an FP32 partial (m, l, o),
//     and the last CTA of its (seq, kv_head) to arrive (threadfence +
//     atomic counter) merges all splits and resets the counter to zero.
#pragma once

#include "common.cuh"
#include "qk_norm_rope.cuh"

namespace rib {
namespace decode {

constexpr int D = 128;
constexpr int TK = 32;                 // keys per pipeline tile
constexpr int NCW = 3;                 // consumer warps
constexpr int SPW = 2;                 // ring slots owned by each consumer warp
constexpr int STAGES = NCW * SPW;      // ring depth
constexpr int NTHREADS = (NCW + 1) * 32;
constexpr int ROW_BYTES = D * 2;       // one key row, BF16
constexpr int kMaxPeers = 8;           // ranks of one NVLink all-gather
constexpr int TILE_BYTES = TK * ROW_BYTES;

constexpr int kMergeSplits = 512;     // splits whose (m, l) the final merge stages in smem

struct Smem {
  alignas(128) uint8_t k[STAGES][TILE_BYTES];
  alignas(128) uint8_t v[STAGES][TILE_BYTES];
  alignas(16) float p[NCW][2][TK];
  alignas(16) float red_o[NCW][2][D];
  float red_m[NCW][2];
  float red_l[NCW][2];
  // merge_m also stages a finished unit's BF16 outputs for the NVLink gather
  // (free by then).  No other buffer fits: with 2 CTAs per SM, the 8.8 KB an
  // SM has left must still hold a GEMV CTA of the next kernel (its input
  // vector), which then starts its weight prefetch beside the decode tail.
  alignas(16) float merge_m[2][kMergeSplits];
  float merge_l[2][kMergeSplits];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  int is_last;
};

struct Params {
  const uint16_t *q;           // [B][nq][128]
  const uint64_t *cache_ptrs;  // [B] device pointers, or null (single cache)
  const uint16_t *cache;       // single [2][nkv][cap][128] cache
  const int32_t *lens;         // [B] device key counts, or null
  int n_single;                // key count when lens == null
  int max_n;                   // host bound on key counts (sizes the grid)
  int cap, nq, nkv;
  int chunk;                   // keys per split, multiple of TK
  int max_splits;
  float qscale;                // scale * log2(e)
  uint16_t *out;               // [B][nq][128]
  float *part_ml;              // [B][nkv][max_splits][2][2]  (m, l)
  float *part_o;               // [B][nkv][max_splits][2][128]
  int *counters;               // [B][nkv]
  int *gcounters;              // [B][nkv][max_groups] first-level merge groups
  int max_groups;              // ceil(max_splits / kMergeGroup)
  const int32_t *caps;         // [B] per-sequence capacities (rows per head), or null: cap
  // All-gather over NVLink (world > 0): the outputs of this rank's heads go
  // straight into every rank's gathered buffer instead of `out`.
  int world, rank, nq_total;
  uint16_t *gout[kMaxPeers];              // per rank: output region of this call
  unsigned long long *gsig[kMaxPeers];    // per rank: signal slots [kMaxPeers]
  unsigned long long epoch;               // > 0, increases by one per call
  int *done;                              // units finalised in this call
  int total_units;
  // Device-side epoch (CUDA-graph replay): when set, the call's epoch is
  // *epoch_dev + 1, gout[] are region bases (region = epoch & 1, region_elems
  // elements each), the last unit stores the epoch back and copies this
  // rank's gathered region into gcopy.
  unsigned long long *epoch_dev;
  size_t region_elems;
  uint16_t *gcopy;
  // Fused norm + RoPE + append (qkv set): q is not read from `q` but formed
  // in each CTA from the new token's projection qkv [B][(nq + 2 nkv) * 128]
  // (per-head RMSNorm with qw, RoPE at position lens[b] - 1), and the CTA
  // whose split holds that position writes the token's K and V rows into the
  // cache first -- the arithmetic of rope::qk_norm_rope_kernel, bit for bit.
  const uint16_t *qkv;
  const uint16_t *qw, *kw;
  float inv_freq[64];   // rope_inv_freq
  // early: lens, caps, cache_ptrs and every cache row
  // below lens[b] - 1 are complete when the kernel starts, so the producer
  // fills the ring with tiles below the new token's row before the
  // programmatic-launch wait; only qkv (and the appended row) come from the
  // kernel launched just before.
  int early;
};


// Final outputs of one (sequence, KV head) unit: res[hh] is dim `tid` of
// query head 2h + hh.  Without gather they go to `out`.  With gather every
// rank's buffer receives them (plain peer stores over NVLink); the rank's
// last unit then publishes the call's epoch to every peer and waits, bounded,
// until every peer's epoch has arrived, so when the kernel ends this rank's
// buffer holds the outputs of all ranks.
__device__ __forceinline__ void finalize_unit(const Params &p, int b, int h, int tid,
                                              const float (&res)[2], int &flag, uint16_t *ostage) {
  if (p.world == 0) {
    if (tid < D) {
      uint16_t *outp = p.out + (static_cast<size_t>(b) * p.nq + 2 * h) * D;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) outp[hh * D + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(res[hh]));
    }
    return;
  }
  // this call's epoch and output region (both fixed on the host, or the
  // region chosen by the epoch read from the device)
  const unsigned long long epoch = p.epoch_dev ? __ldcg(p.epoch_dev) + 1 : p.epoch;
  const size_t region = p.epoch_dev ? (epoch & 1ull) * p.region_elems : 0;
  // Both heads' 512 bytes go to every rank as 16-byte stores (32 per rank),
  // not one 2-byte NVLink write per element.
  if (tid < D) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) ostage[hh * D + tid] = __bfloat16_as_ushort(__float2bfloat16_rn(res[hh]));
  }
  __syncthreads();
  {
    const size_t row = static_cast<size_t>(b) * p.nq_total + p.rank * p.nq + 2 * h;
    for (int k = tid; k < p.world * 32; k += NTHREADS) {
      const int r = k >> 5, i = k & 31;
      *reinterpret_cast<uint4 *>(p.gout[r] + region + row * D + 8 * i) =
          *reinterpret_cast<const uint4 *>(ostage + 8 * i);
    }
  }
  __syncthreads();
  // One system-scope fence after the barrier orders every thread's peer
  // stores (fences are cumulative over what the barrier ordered before them).
  if (tid == 0) {
    __threadfence_system();
    flag = (atomicAdd(p.done, 1) == p.total_units - 1);
  }
  __syncthreads();
  if (!flag) return;
  // last unit of this rank: signal every peer, then wait for every peer
  if (tid == 0) __threadfence_system();
  __syncthreads();
  if (tid < p.world) st_release_sys(p.gsig[tid] + p.rank, epoch);
  if (tid < p.world) {
    const unsigned long long *slot = p.gsig[p.rank] + tid;
    if (ld_acquire_sys(slot) < epoch) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_sys(slot) < epoch) {
        if (global_timer_ns() - t0 > wait_limit_ns()) {
          record_timeout();
          break;
        }
      }
    }
  }
  __syncthreads();
  if (p.epoch_dev) {
    // every rank's outputs are in this rank's region: copy them to the fixed buffer
    const size_t n16 = static_cast<size_t>(p.total_units / p.nkv) * p.nq_total * D / 8;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.gout[p.rank] + region);
    for (size_t i = tid; i < n16; i += NTHREADS) reinterpret_cast<uint4 *>(p.gcopy)[i] = __ldcg(src + i);
    __syncthreads();
    if (tid == 0) *p.epoch_dev = epoch;
  }
  if (tid == 0) *p.done = 0;  // ready for the next call
}

__device__ __forceinline__ void unpack8(const uint4 &r, float *f) {
  f[0] = bf16lo(r.x); f[1] = bf16hi(r.x);
  f[2] = bf16lo(r.y); f[3] = bf16hi(r.y);
  f[4] = bf16lo(r.z); f[5] = bf16hi(r.z);
  f[6] = bf16lo(r.w); f[7] = bf16hi(r.w);
}

// q of KV head h's two query heads for sequence b, pre-scaled: lane (g, j)
// holds dims [8j, 8j+8) and [64+8j, 64+8j+8).
__device__ __forceinline__ void load_q(const Params &p, int b, int h, int lane, float (&qa)[2][16]) {
  const int j = lane & 7;
  const uint16_t *qb = p.q + (static_cast<size_t>(b) * p.nq + 2 * h) * D;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    // L2-coherent loads: in the persistent decode step another CTA wrote q
    // earlier in the same kernel (a line left in this SM's L1 could be stale).
    const uint4 r0 = __ldcg(reinterpret_cast<const uint4 *>(qb + hh * D + 8 * j));
    const uint4 r1 = __ldcg(reinterpret_cast<const uint4 *>(qb + hh * D + 64 + 8 * j));
    unpack8(r0, &qa[hh][0]);
    unpack8(r1, &qa[hh][8]);
#pragma unroll
    for (int d = 0; d < 16; ++d) qa[hh][d] *= p.qscale;
  }
}

// Scores, online softmax and P.V of one ring tile of `rows` keys for both
// query heads of a consumer warp (lane layout described at the top of this
// file); ends with the warp converged, before the slot is released.
__device__ __forceinline__ void consume_tile(const uint8_t *Kt, const uint8_t *Vt, float (&pbuf)[2][TK], int lane,
                                             int rows, const float (&qa)[2][16], float (&m_run)[2],
                                             float (&l_run)[2], float (&o)[2][4]) {
  const int g = lane >> 3, j = lane & 7;

  // ---- scores: group g handles keys g*8 .. g*8+7 of the tile
  float s0[8], s1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint8_t *row = Kt + (g * 8 + i) * ROW_BYTES;
    float kf[16];
    unpack8(*reinterpret_cast<const uint4 *>(row + 16 * j), &kf[0]);
    unpack8(*reinterpret_cast<const uint4 *>(row + 128 + 16 * j), &kf[8]);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      a0 = fmaf(qa[0][d], kf[d], a0);
      a1 = fmaf(qa[1][d], kf[d], a1);
    }
    s0[i] = a0;
    s1[i] = a1;
  }
  // ---- butterfly reduce-scatter over the 8 lanes of the group
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const bool up = j & 4;
    const float snd0 = up ? s0[r] : s0[r + 4], kp0 = up ? s0[r + 4] : s0[r];
    const float snd1 = up ? s1[r] : s1[r + 4], kp1 = up ? s1[r + 4] : s1[r];
    s0[r] = kp0 + __shfl_xor_sync(0xffffffffu, snd0, 4);
    s1[r] = kp1 + __shfl_xor_sync(0xffffffffu, snd1, 4);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const bool up = j & 2;
    const float snd0 = up ? s0[r] : s0[r + 2], kp0 = up ? s0[r + 2] : s0[r];
    const float snd1 = up ? s1[r] : s1[r + 2], kp1 = up ? s1[r + 2] : s1[r];
    s0[r] = kp0 + __shfl_xor_sync(0xffffffffu, snd0, 2);
    s1[r] = kp1 + __shfl_xor_sync(0xffffffffu, snd1, 2);
  }
  {
    const bool up = j & 1;
    const float snd0 = up ? s0[0] : s0[1], kp0 = up ? s0[1] : s0[0];
    const float snd1 = up ? s1[0] : s1[1], kp1 = up ? s1[1] : s1[0];
    s0[0] = kp0 + __shfl_xor_sync(0xffffffffu, snd0, 1);
    s1[0] = kp1 + __shfl_xor_sync(0xffffffffu, snd1, 1);
  }
  // lane l now holds the scores of key l of the tile
  float sc0 = lane < rows ? s0[0] : -INFINITY;
  float sc1 = lane < rows ? s1[0] : -INFINITY;
  float mt0 = sc0, mt1 = sc1;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
    mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
  }
  const float mn0 = fmaxf(m_run[0], mt0), mn1 = fmaxf(m_run[1], mt1);
  const float al0 = fast_exp2(m_run[0] - mn0), al1 = fast_exp2(m_run[1] - mn1);
  m_run[0] = mn0;
  m_run[1] = mn1;
  const float p0 = fast_exp2(sc0 - mn0), p1 = fast_exp2(sc1 - mn1);
  l_run[0] = l_run[0] * al0 + p0;
  l_run[1] = l_run[1] * al1 + p1;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    o[0][e] *= al0;
    o[1][e] *= al1;
  }
  pbuf[0][lane] = p0;
  pbuf[1][lane] = p1;
  __syncwarp();

  // ---- P.V: lane owns dims [4*lane, 4*lane+4)
  int kk = 0;
  for (; kk + 4 <= rows; kk += 4) {
    const float4 pa = *reinterpret_cast<const float4 *>(&pbuf[0][kk]);
    const float4 pb = *reinterpret_cast<const float4 *>(&pbuf[1][kk]);
    const float pa_[4] = {pa.x, pa.y, pa.z, pa.w};
    const float pb_[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint2 vr = *reinterpret_cast<const uint2 *>(Vt + (kk + u) * ROW_BYTES + 8 * lane);
      const float v0 = bf16lo(vr.x), v1 = bf16hi(vr.x), v2 = bf16lo(vr.y), v3 = bf16hi(vr.y);
      o[0][0] = fmaf(pa_[u], v0, o[0][0]);
      o[0][1] = fmaf(pa_[u], v1, o[0][1]);
      o[0][2] = fmaf(pa_[u], v2, o[0][2]);
      o[0][3] = fmaf(pa_[u], v3, o[0][3]);
      o[1][0] = fmaf(pb_[u], v0, o[1][0]);
      o[1][1] = fmaf(pb_[u], v1, o[1][1]);
      o[1][2] = fmaf(pb_[u], v2, o[1][2]);
      o[1][3] = fmaf(pb_[u], v3, o[1][3]);
    }
  }
  for (; kk < rows; ++kk) {
    const float pa = pbuf[0][kk], pb = pbuf[1][kk];
    const uint2 vr = *reinterpret_cast<const uint2 *>(Vt + kk * ROW_BYTES + 8 * lane);
    const float v0 = bf16lo(vr.x), v1 = bf16hi(vr.x), v2 = bf16lo(vr.y), v3 = bf16hi(vr.y);
    o[0][0] = fmaf(pa, v0, o[0][0]);
    o[0][1] = fmaf(pa, v1, o[0][1]);
    o[0][2] = fmaf(pa, v2, o[0][2]);
    o[0][3] = fmaf(pa, v3, o[0][3]);
    o[1][0] = fmaf(pb, v0, o[1][0]);
    o[1][1] = fmaf(pb, v1, o[1][1]);
    o[1][2] = fmaf(pb, v2, o[1][2]);
    o[1][3] = fmaf(pb, v3, o[1][3]);
  }
}

constexpr int kMergeGroup = 16;  // splits per first-level merge group
#ifndef RIB_DECODE_TWO_LEVEL_ABOVE
#define RIB_DECODE_TWO_LEVEL_ABOVE 64  // splits above which the merge takes two levels (build-time tuning)
#endif

// Merges `count` partials (m, l, o) of `unit` held at split slots first,
// first + stride, ...: per head the largest m (M), and l and o weighted by
// exp2(m - M), summed in split order (L, O); thread tid < D computes dim tid.
// The o loads of the first kMergeBatch partials of both heads are issued
// before the (m, l) pairs are staged in shared memory (count <=
// kMergeSplits), so the merge costs one L2 round trip per kMergeBatch
// partials instead of one per head and per unrolled chunk.
#ifndef RIB_DECODE_MERGE_BATCH
#define RIB_DECODE_MERGE_BATCH 40  // partials per merge round trip (build-time tuning)
#endif
constexpr int kMergeBatch = RIB_DECODE_MERGE_BATCH;
__device__ __forceinline__ void merge_partials(const Params &p, Smem &s, size_t unit, int first, int stride,
                                               int count, int tid, float (&M)[2], float (&L)[2], float (&O)[2]) {
  const float *ml = p.part_ml + unit * p.max_splits * 4;  // [split][head][m, l]
  const float *po = p.part_o + unit * p.max_splits * 2 * D;
  float v[2][kMergeBatch];
  auto load_batch = [&](int k0) {
#pragma unroll
    for (int u = 0; u < kMergeBatch; ++u)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
        v[hh][u] = (tid < D && k0 + u < count) ? __ldcg(&po[((first + (k0 + u) * stride) * 2 + hh) * D + tid]) : 0.f;
  };
  load_batch(0);  // in flight while the (m, l) pairs are staged
  for (int i = tid; i < 2 * count; i += NTHREADS) {
    const int k = i >> 1, hh = i & 1;
    const float2 w = __ldcg(reinterpret_cast<const float2 *>(ml) + (first + k * stride) * 2 + hh);
    s.merge_m[hh][k] = w.x;
    s.merge_l[hh][k] = w.y;
  }
  __syncthreads();
  if (tid < D) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float m = -INFINITY;
      for (int k = 0; k < count; ++k) m = fmaxf(m, s.merge_m[hh][k]);
      M[hh] = m;
      L[hh] = 0.f;
      O[hh] = 0.f;
    }
    for (int k0 = 0; k0 < count; k0 += kMergeBatch) {
      if (k0 > 0) load_batch(k0);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) {
          const int k = k0 + u;
          if (k < count) {
            const float f = fast_exp2(s.merge_m[hh][k] - M[hh]);
            L[hh] = fmaf(s.merge_l[hh][k], f, L[hh]);
            O[hh] = fmaf(v[hh][u], f, O[hh]);
          }
        }
    }
  }
}

// q of a CTA's two query heads from shared memory (staged by the fused
// norm + RoPE prologue), with the lane layout and scaling of load_q.
__device__ __forceinline__ void load_q_staged(const uint16_t *qs, float qscale, int lane, float (&qa)[2][16]) {
  const int j = lane & 7;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    unpack8(*reinterpret_cast<const uint4 *>(qs + hh * D + 8 * j), &qa[hh][0]);
    unpack8(*reinterpret_cast<const uint4 *>(qs + hh * D + 64 + 8 * j), &qa[hh][8]);
#pragma unroll
    for (int d = 0; d < 16; ++d) qa[hh][d] *= qscale;
  }
}

// One CTA's work unit: split `split` of KV head h of sequence b.  Used by
// decode_kernel (one unit per CTA) and by the persistent decode-step kernel
// (decode_step.cuh), which calls it with the unit it owns in that phase.
// All NTHREADS threads enter; returns are CTA-uniform.
__device__ __forceinline__ void decode_cta(const Params &p, Smem &s, int split, int h, int b, bool early = false) {
  const int n = p.lens ? p.lens[b] : p.n_single;
  const int cap = p.caps ? p.caps[b] : p.cap;  // rows per head of this sequence's cache
  if (n < 1 || n > cap || n > p.max_n) {  // bad device-side length: record, write nothing
    if (threadIdx.x == 0 && split == 0) atomicExch(&g_device_status, RIB_EINVAL);
    return;
  }
  const int nsplit = (n + p.chunk - 1) / p.chunk;
  if (split >= nsplit) return;  // whole CTA: this sequence needs fewer splits
  const int k_begin = split * p.chunk;
  const int k_end = min(n, k_begin + p.chunk);
  const int ntiles = (k_end - k_begin + TK - 1) / TK;
  const uint16_t *cache = p.cache_ptrs ? reinterpret_cast<const uint16_t *>(p.cache_ptrs[b]) : p.cache;
  if (reinterpret_cast<uintptr_t>(cache) & 15u) {  // bulk copies need 16-byte alignment
    if (threadIdx.x == 0 && split == 0) atomicExch(&g_device_status, RIB_EALIGN);
    return;
  }
  const uint16_t *Kh = cache + static_cast<size_t>(h) * cap * D;
  const uint16_t *Vh = cache + static_cast<size_t>(p.nkv + h) * cap * D;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    fence_mbar_init();
  }
  // Early start: tiles that end below the new token's row do not depend on the
  // kernel before this one; one ring's worth is in flight before the wait.
  const int pre = early ? max(0, min(min(STAGES, ntiles), (n - 1 - k_begin) / TK)) : 0;
  // Fused prologue: the merge buffers are free until the merge, so they hold
  // the RoPE angles and the staged q meanwhile.  The angles depend only on
  // the position n - 1, so with early they are formed before the wait.
  float *cos_t = &s.merge_m[0][0], *sin_t = &s.merge_m[0][64];
  uint16_t *qstage = reinterpret_cast<uint16_t *>(&s.merge_m[1][0]);
  if (early) {
    if (p.qkv) rope::rope_angles(n - 1, p.inv_freq, cos_t, sin_t, tid);
    __syncthreads();  // barriers initialised
    if (warp == NCW && lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      for (int t = 0; t < pre; ++t) {  // t < STAGES: every slot is free, no empty wait
        const int slot = (t % NCW) * SPW + (t / NCW) % SPW;
        const int k0 = k_begin + t * TK;
        const uint32_t bytes = static_cast<uint32_t>(min(TK, k_end - k0)) * ROW_BYTES;
        mbar_arrive_expect_tx(&s.full[slot], 2 * bytes);
        bulk_g2s(s.k[slot], Kh + static_cast<size_t>(k0) * D, bytes, &s.full[slot], pol);
        bulk_g2s(s.v[slot], Vh + static_cast<size_t>(k0) * D, bytes, &s.full[slot], pol);
      }
    }
    pdl_wait();
  }
  if (p.qkv) {
    if (!early) rope::rope_angles(n - 1, p.inv_freq, cos_t, sin_t, tid);
    __syncthreads();
    const int j = lane & 15, half = lane >> 4;
    const unsigned half_mask = 0xffffu << (lane & 16);
    const uint16_t *row = p.qkv + static_cast<size_t>(b) * (p.nq + 2 * p.nkv) * D;
    if (warp == 0) {  // query heads 2h (lanes 0-15) and 2h + 1 (lanes 16-31)
      const uint4 raw = *reinterpret_cast<const uint4 *>(row + (2 * h + half) * D + 8 * j);
      *reinterpret_cast<uint4 *>(qstage + half * D + 8 * j) = rope::norm_rope8(raw, p.qw, j, half_mask, cos_t, sin_t);
    } else if (warp == 1 && k_end == n) {  // the split holding the new token appends its K and V rows
      const uint4 raw = *reinterpret_cast<const uint4 *>(row + (half ? p.nq + p.nkv + h : p.nq + h) * D + 8 * j);
      const uint4 val = half ? raw : rope::norm_rope8(raw, p.kw, j, half_mask, cos_t, sin_t);
      uint16_t *dst = const_cast<uint16_t *>(half ? Vh : Kh) + static_cast<size_t>(n - 1) * D + 8 * j;
      *reinterpret_cast<uint4 *>(dst) = val;
      fence_proxy_async_global();  // the row is read back by this CTA's bulk copies
    }
  }
  __syncthreads();

  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};

  if (warp == NCW) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      for (int t = pre; t < ntiles; ++t) {
        const int k = t / NCW;  // k-th tile of consumer warp t % NCW
        const int slot = (t % NCW) * SPW + k % SPW;
        if (k >= SPW && !mbar_wait(&s.empty[slot], ((k / SPW) - 1) & 1)) break;
        const int k0 = k_begin + t * TK;
        const uint32_t bytes = static_cast<uint32_t>(min(TK, k_end - k0)) * ROW_BYTES;
        mbar_arrive_expect_tx(&s.full[slot], 2 * bytes);
        bulk_g2s(s.k[slot], Kh + static_cast<size_t>(k0) * D, bytes, &s.full[slot], pol);
        bulk_g2s(s.v[slot], Vh + static_cast<size_t>(k0) * D, bytes, &s.full[slot], pol);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    float qa[2][16];
    if (p.qkv)
      load_q_staged(qstage, p.qscale, lane, qa);
    else
      load_q(p, b, h, lane, qa);
    for (int t = warp, k = 0; t < ntiles; t += NCW, ++k) {
      const int slot = warp * SPW + k % SPW;
      if (!mbar_wait(&s.full[slot], (k / SPW) & 1)) break;
      const int k0 = k_begin + t * TK;
      consume_tile(s.k[slot], s.v[slot], s.p[warp], lane, min(TK, k_end - k0), qa, m_run, l_run, o);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[slot]);
    }
    // ---- publish this warp's state
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float l = l_run[hh];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) {
        s.red_m[warp][hh] = m_run[hh];
        s.red_l[warp][hh] = l;
      }
      *reinterpret_cast<float4 *>(&s.red_o[warp][hh][4 * lane]) =
          make_float4(o[hh][0], o[hh][1], o[hh][2], o[hh][3]);
    }
  }
  __syncthreads();

  // ------------------------------------------------------------ CTA merge
  // threads 0..127: dim d = tid, both heads.
  float Mx[2] = {-INFINITY, -INFINITY}, Lx[2] = {0.f, 0.f}, Ox[2] = {0.f, 0.f};
  if (tid < D) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NCW; ++w) M = fmaxf(M, s.red_m[w][hh]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        const float mw = s.red_m[w][hh];
        const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
        L = fmaf(s.red_l[w][hh], f, L);
        O = fmaf(s.red_o[w][hh][tid], f, O);
      }
      Mx[hh] = M;
      Lx[hh] = L;
      Ox[hh] = O;
    }
  }
  float res[2] = {0.f, 0.f};
  if (nsplit == 1) {
    if (tid < D) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) res[hh] = Ox[hh] / Lx[hh];
    }
    finalize_unit(p, b, h, tid, res, s.is_last, reinterpret_cast<uint16_t *>(&s.merge_m[0][0]));
    return;
  }
  const size_t unit = static_cast<size_t>(b) * p.nkv + h;
  if (tid < D) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const size_t pi = (unit * p.max_splits + split) * 2 + hh;
      p.part_o[pi * D + tid] = Ox[hh];
      if (tid == 0) {
        p.part_ml[pi * 2 + 0] = Mx[hh];
        p.part_ml[pi * 2 + 1] = Lx[hh];
      }
    }
  }
  __threadfence();
  __syncthreads();
  // Two-level merge: above RIB_DECODE_TWO_LEVEL_ABOVE splits, the last CTA of
  // each group of kMergeGroup consecutive splits merges the group into the
  // slot of its first split, and the last group merges the group results;
  // one CTA merging hundreds of partials would spend tens of microseconds in
  // dependent L2 round trips at the end of the launch.  For few splits one
  // level is faster (the second level adds an atomic round trip).
  const int ngroups = nsplit > RIB_DECODE_TWO_LEVEL_ABOVE ? (nsplit + kMergeGroup - 1) / kMergeGroup : 1;
  int first = 0, stride = 1, count = nsplit;
  if (ngroups > 1) {
    const int g = split / kMergeGroup, g0 = g * kMergeGroup, gn = min(kMergeGroup, nsplit - g0);
    int *gc = p.gcounters + unit * p.max_groups + g;
    if (tid == 0) s.is_last = (atomicAdd(gc, 1) == gn - 1);
    __syncthreads();
    if (!s.is_last) return;
    __threadfence();
    float M[2], L[2], O[2];
    merge_partials(p, s, unit, g0, 1, gn, tid, M, L, O);
    if (tid < D) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const size_t pi = (unit * p.max_splits + g0) * 2 + hh;
        p.part_o[pi * D + tid] = O[hh];
        if (tid == 0) {
          p.part_ml[pi * 2 + 0] = M[hh];
          p.part_ml[pi * 2 + 1] = L[hh];
        }
      }
    }
    if (tid == 0) *gc = 0;  // leave the workspace ready for the next call
    __threadfence();
    __syncthreads();
    stride = kMergeGroup;
    count = ngroups;
  }
  if (tid == 0) s.is_last = (atomicAdd(&p.counters[unit], 1) == count - 1);
  __syncthreads();
  if (!s.is_last) return;
  __threadfence();
  {
    float M[2], L[2], O[2];
    merge_partials(p, s, unit, first, stride, count, tid, M, L, O);
    if (tid < D) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) res[hh] = O[hh] / L[hh];
    }
  }
  if (tid == 0) p.counters[unit] = 0;  // leave the workspace ready for the next call
  __syncthreads();
  finalize_unit(p, b, h, tid, res, s.is_last, reinterpret_cast<uint16_t *>(&s.merge_m[0][0]));
}

__global__ void __launch_bounds__(NTHREADS, 2) decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  pdl_launch_dependents();
  if (!p.early) pdl_wait();  // (with early, decode_cta waits after its first bulk copies)
  decode_cta(p, s, blockIdx.x, blockIdx.y, blockIdx.z, p.early != 0);
}

}  // namespace decode
}  // namespace rib
