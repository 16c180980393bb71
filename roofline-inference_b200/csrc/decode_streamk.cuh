// Stream-K split-KV decode: the decode of decode_attention.cuh with its work
// cut evenly over one wave of CTAs instead of into fixed-size splits.
//
// Every (sequence b, KV head h) unit is a run of ceil(n_b / TK) key tiles;
// the units of a launch are laid end to end (sequence-major, head-minor) and
// CTA c of G takes tiles [c * tpc, (c + 1) * tpc), tpc = max(ceil(T / G),
// kStreamMinTiles), T the total.  A CTA therefore works through one or more
// segments (the part of a unit inside its range): the producer warp streams
// the tiles of all its segments through the ring without a break, the three
// consumer warps take tiles round-robin as in the split kernel and, at the end
// of each segment, merge their states among themselves (named barrier 1 of 96
// threads; the producer warp runs ahead).  A segment that is a whole unit is
// written out directly; otherwise it leaves an FP32 partial (m, l, o) in slot
// `c - first CTA of the unit`, and the last segment of the unit to arrive
// (atomic counter) merges them.  With all CTAs resident at once there is no
// partly filled last wave, and the per-CTA start-up is paid once per SM slot,
// not once per split.
#pragma once

#include "decode_attention.cuh"

namespace rib {
namespace decode {

constexpr int kStreamMinTiles = 16;    // fewest tiles per CTA (bounds segments per unit)
constexpr int kStreamMaxSeqs = 256;    // sequences per launch (tile prefix kept in shared memory)
constexpr int kStreamMaxSegs = 320;    // segments per unit: at most one wave of CTAs (2 x 148) + 1
constexpr int NCT = NCW * 32;          // consumer threads
constexpr int kStreamMergeBatch = 16;  // segments whose partial outputs one merge round trip loads

struct StreamSmem {
  alignas(128) uint8_t k[STAGES][TILE_BYTES];
  alignas(128) uint8_t v[STAGES][TILE_BYTES];
  alignas(16) float p[NCW][2][TK];
  alignas(16) float red_o[NCW][2][D];  // red_o[0] also holds a finished unit's results
  float red_m[NCW][2];
  float red_l[NCW][2];
  alignas(16) float merge_m[2][kStreamMaxSegs];  // also stages a finished unit's BF16 outputs
  float merge_l[2][kStreamMaxSegs];
  int pre[kStreamMaxSeqs + 1];  // tiles before sequence b, all its heads included
  int scan[NTHREADS];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  int is_last;
};

// Segments a unit of at most max_n keys can be cut into.
__host__ __device__ constexpr int stream_max_segments(int max_n) {
  return ((max_n + TK - 1) / TK + kStreamMinTiles - 1) / kStreamMinTiles + 1;
}

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(NCT) : "memory");
}

// Unit of global tile t: sequence b (largest with pre[b] <= t), head h, the
// unit's first tile [ustart, uend) and the sequence's key count n.
struct UnitPos {
  int b, h, ustart, uend;
};

__device__ __forceinline__ UnitPos locate(const StreamSmem &s, int B, int nkv, int t) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {  // largest b with pre[b] <= t (sequences with no tiles share a prefix value)
    const int mid = (lo + hi + 1) >> 1;
    if (s.pre[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  const int per_head = (s.pre[lo + 1] - s.pre[lo]) / nkv;
  const int h = (t - s.pre[lo]) / per_head;
  UnitPos u;
  u.b = lo;
  u.h = h;
  u.ustart = s.pre[lo] + h * per_head;
  u.uend = u.ustart + per_head;
  return u;
}

// Output of one finished unit (s.red_o[0]) for the 96 consumer threads:
// plain stores, or the NVLink all-gather of finalize_unit
// (decode_attention.cuh) without its completion step.  A CTA may finish a
// unit in the middle of its run of tiles, so the system-scope fence that
// makes the peer stores visible, the count of finished units and the last
// unit's signal and wait are deferred to stream_gather_done at the CTA's end:
// one fence per CTA, and none in the middle of its streaming.
__device__ __forceinline__ void stream_finalize(const Params &p, StreamSmem &s, int b, int h, int ct) {
  if (p.world == 0) {
    uint16_t *outp = p.out + (static_cast<size_t>(b) * p.nq + 2 * h) * D;
    for (int i = ct; i < 2 * D; i += NCT) outp[i] = __bfloat16_as_ushort(__float2bfloat16_rn(s.red_o[0][i >> 7][i & 127]));
    return;
  }
  const unsigned long long epoch = p.epoch_dev ? __ldcg(p.epoch_dev) + 1 : p.epoch;
  const size_t region = p.epoch_dev ? (epoch & 1ull) * p.region_elems : 0;
  const size_t row = static_cast<size_t>(b) * p.nq_total + p.rank * p.nq + 2 * h;
  uint16_t *ostage = reinterpret_cast<uint16_t *>(&s.merge_m[0][0]);  // free once the unit is merged
  for (int i = ct; i < 2 * D; i += NCT) ostage[i] = __bfloat16_as_ushort(__float2bfloat16_rn(s.red_o[0][i >> 7][i & 127]));
  consumer_sync();
  for (int k = ct; k < p.world * 32; k += NCT) {  // 16-byte NVLink stores, 32 per rank
    const int r = k >> 5, i = k & 31;
    *reinterpret_cast<uint4 *>(p.gout[r] + region + row * D + 8 * i) = *reinterpret_cast<const uint4 *>(ostage + 8 * i);
  }
}

// End of a gathering CTA that finished `fin` units: one system-scope fence
// after the barrier orders every thread's peer stores, then the units count
// towards the rank's total; the CTA that completes it signals every peer and
// waits, bounded, for every peer's signal, so when the kernel ends this
// rank's buffer holds the outputs of all ranks.
__device__ __forceinline__ void stream_gather_done(const Params &p, StreamSmem &s, int ct, int fin) {
  consumer_sync();
  if (ct == 0) {
    bool last = false;
    if (fin > 0) {
      __threadfence_system();
      last = atomicAdd(p.done, fin) + fin == p.total_units;
    }
    s.is_last = last;
  }
  consumer_sync();
  if (!s.is_last) return;
  const unsigned long long epoch = p.epoch_dev ? __ldcg(p.epoch_dev) + 1 : p.epoch;
  const size_t region = p.epoch_dev ? (epoch & 1ull) * p.region_elems : 0;
  if (ct == 0) __threadfence_system();
  consumer_sync();
  if (ct < p.world) st_release_sys(p.gsig[ct] + p.rank, epoch);
  if (ct < p.world) {
    const unsigned long long *slot = p.gsig[p.rank] + ct;
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
  consumer_sync();
  if (p.epoch_dev) {
    const size_t n16 = static_cast<size_t>(p.total_units / p.nkv) * p.nq_total * D / 8;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.gout[p.rank] + region);
    for (size_t i = ct; i < n16; i += NCT) reinterpret_cast<uint4 *>(p.gcopy)[i] = __ldcg(src + i);
    consumer_sync();
    if (ct == 0) *p.epoch_dev = epoch;
  }
  if (ct == 0) *p.done = 0;  // ready for the next call
}

__global__ void __launch_bounds__(NTHREADS, 2) decode_streamk_kernel(const __grid_constant__ Params p, int B) {
  extern __shared__ uint8_t smem_raw[];
  StreamSmem &s =
      *reinterpret_cast<StreamSmem *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  pdl_launch_dependents();
  // With early, lens, caps, cache_ptrs and every cache row below lens[b] - 1
  // are complete when the kernel starts: the prefix scan and the producer's
  // first ring of such tiles run before the programmatic-launch wait.
  if (!p.early) pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- tiles per sequence (all heads), exclusive prefix over sequences.
  // Thread t counts a contiguous run of at most kStreamMaxSeqs / NTHREADS
  // sequences, the CTA scans the NTHREADS sums, thread t writes its run's
  // prefixes.
  constexpr int kPer = kStreamMaxSeqs / NTHREADS;
  const int per = (B + NTHREADS - 1) / NTHREADS;  // <= kPer (checked on the host)
  const int b0 = tid * per, b1 = min(B, b0 + per);
  int cnt[kPer];
  int mine = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int b = b0 + i;
    cnt[i] = 0;
    if (b >= b1) continue;
    const int n = p.lens ? p.lens[b] : p.n_single;
    const int cap = p.caps ? p.caps[b] : p.cap;
    int tiles = (n + TK - 1) / TK;
    if (n < 1 || n > cap || n > p.max_n) {  // bad device-side length: record, no work
      if (blockIdx.x == 0) atomicExch(&g_device_status, RIB_EINVAL);
      tiles = 0;
    } else if (p.cache_ptrs && (p.cache_ptrs[b] & 15u)) {  // bulk copies need 16-byte alignment
      if (blockIdx.x == 0) atomicExch(&g_device_status, RIB_EALIGN);
      tiles = 0;
    }
    cnt[i] = tiles * p.nkv;
    mine += cnt[i];
  }
  s.scan[tid] = mine;
  __syncthreads();
  if (warp == 0) {  // exclusive scan of the NTHREADS sums, NTHREADS / 32 per lane
    constexpr int kLane = NTHREADS / 32;
    int v[kLane], run = 0;
#pragma unroll
    for (int i = 0; i < kLane; ++i) {
      v[i] = run;
      run += s.scan[lane * kLane + i];
    }
    int incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    const int base = incl - run;
#pragma unroll
    for (int i = 0; i < kLane; ++i) s.scan[lane * kLane + i] = base + v[i];
    if (lane == 31) s.pre[B] = incl;  // total tiles
  }
  __syncthreads();
  {
    int run = s.scan[tid];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      if (b0 + i >= b1) break;
      s.pre[b0 + i] = run;
      run += cnt[i];
    }
  }
  __syncthreads();
  const int T = s.pre[B];
  const int G = gridDim.x;
  const int tpc = max((T + G - 1) / G, kStreamMinTiles);
  const int t_begin = blockIdx.x * tpc;
  const int t_end = min(T, t_begin + tpc);
  if (t_begin >= t_end) {  // CTA-uniform
    if (p.early) pdl_wait();
    return;
  }

  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    const uint64_t pol = l2_policy_evict_first();
    UnitPos u = locate(s, B, p.nkv, t_begin);
    const uint16_t *Kh = nullptr, *Vh = nullptr;
    int n = 0;
    bool fresh = true;
    bool waited = !p.early;
    for (int t = t_begin; t < t_end; ++t) {
      if (t >= u.uend) {
        u = locate(s, B, p.nkv, t);
        fresh = true;
      }
      if (fresh) {
        const uint16_t *cache = p.cache_ptrs ? reinterpret_cast<const uint16_t *>(p.cache_ptrs[u.b]) : p.cache;
        const int cap = p.caps ? p.caps[u.b] : p.cap;
        n = p.lens ? p.lens[u.b] : p.n_single;
        Kh = cache + static_cast<size_t>(u.h) * cap * D;
        Vh = cache + static_cast<size_t>(p.nkv + u.h) * cap * D;
        fresh = false;
      }
      const int g = t - t_begin, k = g / NCW;
      const int slot = (g % NCW) * SPW + k % SPW;
      const int k0 = (t - u.ustart) * TK;
      // early: a full ring, and only tiles that end below the new token's row,
      // go out before the wait
      if (!waited && (g >= STAGES || k0 + TK > n - 1)) {
        pdl_wait();
        waited = true;
      }
      if (k >= SPW && !mbar_wait(&s.empty[slot], ((k / SPW) - 1) & 1)) return;
      const uint32_t bytes = static_cast<uint32_t>(min(TK, n - k0)) * ROW_BYTES;
      mbar_arrive_expect_tx(&s.full[slot], 2 * bytes);
      bulk_g2s(s.k[slot], Kh + static_cast<size_t>(k0) * D, bytes, &s.full[slot], pol);
      bulk_g2s(s.v[slot], Vh + static_cast<size_t>(k0) * D, bytes, &s.full[slot], pol);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  if (p.early) pdl_wait();  // q and the outputs' readers belong to the previous kernel
  const int ct = tid;  // 0 .. NCT-1
  int kw = 0;          // tiles this warp has consumed (ring position)
  bool dead = false;   // a wait gave up: skip the remaining waits
  int fin = 0;         // units this CTA finished (all-gather count)
  for (int seg = t_begin; seg < t_end;) {
    const UnitPos u = locate(s, B, p.nkv, seg);
    const int seg_end = min(t_end, u.uend);
    const int n = p.lens ? p.lens[u.b] : p.n_single;
    float qa[2][16];
    load_q(p, u.b, u.h, lane, qa);
    float m_run[2] = {-INFINITY, -INFINITY};
    float l_run[2] = {0.f, 0.f};
    float o[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    // this warp's tiles of the segment: global g = t - t_begin with g % NCW == warp
    const int g0 = seg - t_begin, g1 = seg_end - t_begin;
    for (int g = g0 + ((warp - g0 % NCW) + NCW) % NCW; g < g1; g += NCW, ++kw) {
      const int slot = warp * SPW + kw % SPW;
      if (!dead && !mbar_wait(&s.full[slot], (kw / SPW) & 1)) dead = true;
      if (dead) continue;
      const int k0 = (t_begin + g - u.ustart) * TK;
      consume_tile(s.k[slot], s.v[slot], s.p[warp], lane, min(TK, n - k0), qa, m_run, l_run, o);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[slot]);
    }
    // ---- publish this warp's state, merge the three warps
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float l = l_run[hh];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
      if (lane == 0) {
        s.red_m[warp][hh] = m_run[hh];
        s.red_l[warp][hh] = l;
      }
      *reinterpret_cast<float4 *>(&s.red_o[warp][hh][4 * lane]) = make_float4(o[hh][0], o[hh][1], o[hh][2], o[hh][3]);
    }
    consumer_sync();
    const bool whole = seg == u.ustart && seg_end == u.uend;
    const int unit = u.b * p.nkv + u.h;
    const int first_cta = u.ustart / tpc;
    const int nseg = (u.uend - 1) / tpc - first_cta + 1;
    const int seg_id = blockIdx.x - first_cta;
    float Mi[3], Li[3], Oi[3];
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      const int i = ct + q * NCT;
      Mi[q] = -INFINITY;
      Li[q] = 0.f;
      Oi[q] = 0.f;
      if (i >= 2 * D) continue;
      const int hh = i >> 7, d = i & 127;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < NCW; ++w) M = fmaxf(M, s.red_m[w][hh]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        const float mw = s.red_m[w][hh];
        const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
        L = fmaf(s.red_l[w][hh], f, L);
        O = fmaf(s.red_o[w][hh][d], f, O);
      }
      Mi[q] = M;
      Li[q] = L;
      Oi[q] = O;
      if (whole) s.red_o[0][hh][d] = O / L;
    }
    bool emit = whole;
    if (!whole) {
      // partial of this segment, then the unit's last segment merges all
      float *ml = p.part_ml + static_cast<size_t>(unit) * p.max_splits * 4;
      float *po = p.part_o + static_cast<size_t>(unit) * p.max_splits * 2 * D;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int i = ct + q * NCT;
        if (i >= 2 * D) continue;
        const int hh = i >> 7, d = i & 127;
        po[(seg_id * 2 + hh) * D + d] = Oi[q];
        if (d == 0) {
          ml[(seg_id * 2 + hh) * 2 + 0] = Mi[q];
          ml[(seg_id * 2 + hh) * 2 + 1] = Li[q];
        }
      }
      __threadfence();
      consumer_sync();
      if (ct == 0) s.is_last = atomicAdd(&p.counters[unit], 1) == nseg - 1;
      consumer_sync();
      emit = s.is_last;
      if (emit) {
        __threadfence();
        // The o loads of the first kStreamMergeBatch segments of all three
        // outputs go out before the (m, l) pairs are staged; each output is
        // summed in segment order.
        float v[3][kStreamMergeBatch];
        auto load_batch = [&](int k0) {
#pragma unroll
          for (int u = 0; u < kStreamMergeBatch; ++u)
#pragma unroll
            for (int q = 0; q < 3; ++q) {
              const int i = ct + q * NCT;
              v[q][u] = (i < 2 * D && k0 + u < nseg) ? __ldcg(&po[((k0 + u) * 2 + (i >> 7)) * D + (i & 127)]) : 0.f;
            }
        };
        load_batch(0);
        for (int i = ct; i < 2 * nseg; i += NCT) {
          const float2 w = __ldcg(reinterpret_cast<const float2 *>(ml) + i);
          s.merge_m[i & 1][i >> 1] = w.x;
          s.merge_l[i & 1][i >> 1] = w.y;
        }
        consumer_sync();
        float M[3], L[3] = {0.f, 0.f, 0.f}, O[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          const int hh = ((ct + q * NCT) >> 7) & 1;
          M[q] = -INFINITY;
          for (int sp = 0; sp < nseg; ++sp) M[q] = fmaxf(M[q], s.merge_m[hh][sp]);
        }
        for (int k0 = 0; k0 < nseg; k0 += kStreamMergeBatch) {
          if (k0 > 0) load_batch(k0);
#pragma unroll
          for (int q = 0; q < 3; ++q) {
            const int hh = ((ct + q * NCT) >> 7) & 1;
#pragma unroll
            for (int u = 0; u < kStreamMergeBatch; ++u) {
              const int sp = k0 + u;
              if (sp < nseg) {
                const float f = fast_exp2(s.merge_m[hh][sp] - M[q]);
                L[q] = fmaf(s.merge_l[hh][sp], f, L[q]);
                O[q] = fmaf(v[q][u], f, O[q]);
              }
            }
          }
        }
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          const int i = ct + q * NCT;
          if (i < 2 * D) s.red_o[0][i >> 7][i & 127] = O[q] / L[q];
        }
        if (ct == 0) p.counters[unit] = 0;  // leave the workspace ready for the next call
      }
    }
    consumer_sync();
    if (emit) {
      stream_finalize(p, s, u.b, u.h, ct);
      ++fin;
    }
    consumer_sync();  // s.res, s.red_* and s.merge_* are reused by the next segment
    seg = seg_end;
  }
  if (p.world > 0) stream_gather_done(p, s, ct, fin);
}

}  // namespace decode
}  // namespace rib
