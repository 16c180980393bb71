// Persistent BF16 GEMM on sm_100a for the Qwen3 prefill projections:
// C[M, N] = epi(A[M, K] * W[N, K]^T), tcgen05.mma with the FP32 accumulator
// in TMEM, both operands staged by TMA.
//
// Replaces the library matmul the reference's engine calls for prompts of
// more than 32 tokens (agent-test/v2/engine.py:95-99: mx.matmul; the
// skinny_gemm of kernels.py:273-334 covers 8 < M <= 32), and fuses what
// follows each projection in Engine.prefill (engine.py:110-135):
//   kBF16    C = bf16(A W^T)                      (O and down projections)
//   kF32     C = A W^T in FP32                    (tensor-parallel partials)
//   kSwiGLU  W = [gate; up] (N = 2F rows); C[M, F] = bf16(bf16(g bf16(sigmoid g)) u)
//            with g = bf16(A Wg^T), u = bf16(A Wu^T)  (engine.py:28-30, 133)
//   kQKRope  W = the QKV projection; per (token, head) tile: per-head RMSNorm
//            and RoPE of q and k with the arithmetic of rope::norm_rope8
//            (kernels.py:116-146, 169-204), Q written to [nq][Lp][128] (pad
//            rows zero), K and V appended to the cache rows pos0 + m
//            (engine.py:111-113): the qkv activations never reach HBM.
//
// CTA (one per SM, persistent over output tiles of 128 x BN, or 256 x 256 as
// two halves when there are enough such tiles to fill the GPU): 6 warps.
//   warp 0      TMA producer: A and W k-blocks of 64 (128-byte swizzle) into
//               an NS-stage ring (4 x 48 KB at BN = 256, 6 x 32 KB at 128,
//               3 x 64 KB for 256-row tiles).
//   warp 1      TMEM owner and MMA issuer: per k-block 4 x tcgen05.mma
//               (M = 128, N = BN, K = 16) per 128-row half, into one of two
//               accumulators for 128-row tiles, so the epilogue of tile i
//               overlaps the main loop of tile i + 1.
//   warps 2-5   epilogue: thread = accumulator row (TMEM lane quadrant
//               warp % 4), tcgen05.ld of 32 columns at a time.
// Every wait is bounded (common.cuh); on a timeout the CTA drains its copies,
// frees TMEM and returns with RIB_ETIMEOUT recorded.  No TMA multicast.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "model_kernels.cuh"
#include "qk_norm_rope.cuh"

namespace rib {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle panel of BF16
constexpr int NWARPS = 6;
constexpr int NTHREADS = NWARPS * 32;
constexpr int kEpiThreads = 128;

enum Epi : int { kBF16 = 0, kF32 = 1, kSwiGLU = 2, kQKRope = 3, kF32Owner = 4 };

constexpr int kMaxRanks = 8;

// MH = 1: 128-row tiles, two accumulators (the epilogue of one tile overlaps
// the next tile's MMAs).  MH = 2: 256-row tiles as two M = 128 halves that
// share every W stage -- 64 KB per k-block for twice the FLOPs of the 48 KB
// of a 128 x 256 tile -- with one accumulator pair filling all 512 TMEM
// columns, so the epilogue does not overlap the next tile's MMAs.
template <int BN, int MH = 1>
struct Cfg {
  static_assert(BN == 128 || BN == 256, "BN is 128 or 256");
  static_assert(MH == 1 || (MH == 2 && BN == 256), "256-row tiles take BN = 256");
  static constexpr int A_HALF = BM * BK * 2;
  static constexpr int A_BYTES = MH * A_HALF;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NS = MH == 2 ? 3 : (BN == 256 ? 4 : 6);
  static constexpr int NBUF = MH == 2 ? 1 : 2;  // accumulator buffers
  static constexpr uint32_t TMEM_COLS = NBUF * MH * BN;
  // kind::f16: D = F32 (bit 4), A = B = BF16 (bits 7, 10), both K-major,
  // N >> 3 at bits 17-22, M >> 4 at bits 24-28.
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) |
                                    (static_cast<uint32_t>(BN >> 3) << 17) |
                                    (static_cast<uint32_t>(BM >> 4) << 24);
};

template <int BN, int MH>
struct Smem {
  alignas(1024) uint8_t stage[Cfg<BN, MH>::NS][Cfg<BN, MH>::STAGE];
  uint64_t full[Cfg<BN, MH>::NS], empty[Cfg<BN, MH>::NS];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  // kF32Owner: each epilogue warp's 32 rows x 32 columns, rows padded to 36
  // floats (16-byte stores and loads without bank conflicts)
  alignas(16) float ostage[4][32 * 36];
};

struct Params {
  CUtensorMap tm_a;   // A [M][K], box (64, 128)
  CUtensorMap tm_b;   // W [N][K], box (64, BN) (kSwiGLU: (64, BN / 2), two loads)
  int M, N, K;
  int num_m, num_tiles;
  int epi;
  void *c;            // kBF16 / kSwiGLU: BF16 [M][ldc]; kF32: FP32 [M][ldc]
  long long ldc;
  int swiglu_f;       // kSwiGLU: F (up rows start at F)
  // kQKRope
  const uint16_t *qw, *kw;  // [128] each
  const float2 *rope;       // [>= num_m * 128][64] (cos, sin) of positions pos0 + m
  int pos0, nq, nkv;
  uint16_t *q_out;          // [nq][Lp][128]
  int Lp;
  uint16_t *cache;          // [2][nkv][cap][128]
  int cap;
  // kF32Owner (tensor-parallel prefill): row m's FP32 partial goes to rank
  // o = m / rpo's receive buffer, slot `rank`, row m - o rpo (a plain store
  // when o is this rank, else a store over NVLink); ldc = N.
  float *owner_recv[kMaxRanks];  // each rank's receive slots [world][rpo_cap][N], as seen from here
  int rpo, rank;
  long long slot_floats;         // rpo_cap * N
};

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  // K-major, 128-byte swizzle (layout 2 at bits 61-63), sm100 version bit 46,
  // LBO 16 B (unused), SBO 1024 B (8 rows of 128 B); addresses in 16-byte units.
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int c0, int c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

template <class S>
__device__ __forceinline__ bool aborted(const S &s) {
  return *reinterpret_cast<const volatile int *>(&s.abort_flag) != 0;
}
template <class S>
__device__ __forceinline__ void set_abort(S &s) {
  *reinterpret_cast<volatile int *>(&s.abort_flag) = 1;
}

__device__ __forceinline__ float silu_bf16(float g) {
  // s = bf16(sigmoid(g)), a = bf16(g s)  (agent-test/v2/kernels.py:86-93),
  // the arithmetic of model::swiglu_kernel
  return round_bf16(g * model::sigmoid_bf16(g));
}

// ---------------------------------------------------------------- epilogues
// Row `m` of the tile's accumulator at TMEM address `ta` (this thread's
// lane, column 0).  All 32 lanes of the warp execute every tcgen05.ld.
template <int BN>
__device__ __forceinline__ void epi_store(const Params &p, uint32_t ta, int m, int n0) {
  const bool row_ok = m < p.M;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    uint32_t r[32];
    tmem_ld32(ta + c0, r);
    tmem_wait_ld();
    const int ncols = p.N - (n0 + c0);  // columns past N (a ragged last tile) are not stored
    if (!row_ok || ncols <= 0) continue;
    if (p.epi == kF32) {
      float4 *dst = reinterpret_cast<float4 *>(static_cast<float *>(p.c) + m * p.ldc + n0 + c0);
#pragma unroll
      for (int v = 0; v < 8; ++v)
        if (4 * v < ncols)
          dst[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                               __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
    } else {
      uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.c) + m * p.ldc + n0 + c0);
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        if (8 * v >= ncols) break;
        uint4 w;
        w.x = pack_bf16x2(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
        w.y = pack_bf16x2(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
        w.z = pack_bf16x2(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
        w.w = pack_bf16x2(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
        dst[v] = w;
      }
    }
  }
}

// kF32Owner: the rows of this warp (m_base + lane) go to their owner ranks.
// A thread holds one row of 32 columns after tcgen05.ld; staged through
// shared memory, each store instruction then writes four rows' 128-byte
// segments (eight lanes per row) instead of 32 scattered 16-byte pieces, the
// form that moves well over NVLink.
template <int BN>
__device__ __forceinline__ void epi_store_owner(const Params &p, uint32_t ta, int m_base, int n0, float *stage) {
  const int lane = threadIdx.x & 31;
  const int j = lane & 7;
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    uint32_t r[32];
    tmem_ld32(ta + c0, r);
    tmem_wait_ld();
    float4 *srow = reinterpret_cast<float4 *>(stage + lane * 36);
#pragma unroll
    for (int v = 0; v < 8; ++v)
      srow[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                            __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
    __syncwarp();
    const int ncols = p.N - (n0 + c0);  // columns past N (a ragged last tile) are not stored
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int i = it * 4 + (lane >> 3);
      const int m = m_base + i;
      if (m < p.M && 4 * j < ncols) {
        const float4 v = *reinterpret_cast<const float4 *>(stage + i * 36 + 4 * j);
        float *row = p.owner_recv[m / p.rpo] + p.rank * p.slot_floats + (m % p.rpo) * p.ldc;
        *reinterpret_cast<float4 *>(row + n0 + c0 + 4 * j) = v;
      }
    }
    __syncwarp();
  }
}

// kSwiGLU (BN = 256): columns [0, 128) are gate rows f0 .. f0 + 127, columns
// [128, 256) the matching up rows; writes C[m, f0 .. f0 + 127].
__device__ __forceinline__ void epi_swiglu(const Params &p, uint32_t ta, int m, int f0) {
  const bool row_ok = m < p.M;
#pragma unroll 1
  for (int c0 = 0; c0 < 128; c0 += 32) {
    uint32_t g[32], u[32];
    tmem_ld32(ta + c0, g);
    tmem_ld32(ta + 128 + c0, u);
    tmem_wait_ld();
    if (!row_ok) continue;
    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(p.c) + m * p.ldc + f0 + c0);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float gg = round_bf16(__uint_as_float(g[8 * v + e]));
        const float uu = round_bf16(__uint_as_float(u[8 * v + e]));
        y[e] = silu_bf16(gg) * uu;
      }
      uint4 w;
      w.x = pack_bf16x2(y[0], y[1]);
      w.y = pack_bf16x2(y[2], y[3]);
      w.z = pack_bf16x2(y[4], y[5]);
      w.w = pack_bf16x2(y[6], y[7]);
      dst[v] = w;
    }
  }
}

// kQKRope: each 128 columns of the tile are one head `h` of the QKV
// projection for 128 tokens (a 256-wide tile holds two heads, done one after
// the other).  The sum of squares is combined in the order rope::norm_rope8 uses
// (eight-element FMA chains per 16-lane group member, then an xor tree), so
// for the same BF16 qkv values the outputs are bit-identical to the
// two-kernel path (GEMM, then qk_norm_rope_append).
__device__ __forceinline__ void epi_qk_rope(const Params &p, uint32_t ta, int m, int h) {
  uint32_t r[128];
#pragma unroll
  for (int c = 0; c < 4; ++c) tmem_ld32(ta + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&r[32 * c]));
  tmem_wait_ld();
  const int nq = p.nq, nkv = p.nkv;
  if (m >= p.M) {
    // Q pad rows [M, Lp) are zero (kernels.py:223, init_value=0)
    if (h < nq && m < p.Lp) {
      uint4 *dst = reinterpret_cast<uint4 *>(p.q_out + (static_cast<size_t>(h) * p.Lp + m) * 128);
#pragma unroll
      for (int v = 0; v < 16; ++v) dst[v] = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  float x[128];
#pragma unroll
  for (int d = 0; d < 128; ++d) x[d] = round_bf16(__uint_as_float(r[d]));  // the BF16 qkv value
  uint16_t *dst;
  if (h >= nq + nkv) {  // V: copied into the cache
    dst = p.cache + ((static_cast<size_t>(nkv + h - nq - nkv) * p.cap) + p.pos0 + m) * 128;
    uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int v = 0; v < 16; ++v) {
      uint4 w;
      w.x = pack_bf16x2(x[8 * v + 0], x[8 * v + 1]);
      w.y = pack_bf16x2(x[8 * v + 2], x[8 * v + 3]);
      w.z = pack_bf16x2(x[8 * v + 4], x[8 * v + 5]);
      w.w = pack_bf16x2(x[8 * v + 6], x[8 * v + 7]);
      d4[v] = w;
    }
    return;
  }
  // sum of squares: 16 chains of 8 (dims [8j, 8j+8)), then the xor tree 8, 4, 2, 1
  float s16[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) a = fmaf(x[8 * j + i], x[8 * j + i], a);
    s16[j] = a;
  }
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1)
#pragma unroll
    for (int j = 0; j < o; ++j) s16[j] = s16[j] + s16[j + o];
  const float inv = 1.0f / sqrtf(s16[0] / 128.0f + 1e-6f);
  const uint16_t *w = h < nq ? p.qw : p.kw;
  float n[128];
#pragma unroll
  for (int v = 0; v < 16; ++v) {
    const uint4 wr = *reinterpret_cast<const uint4 *>(w + 8 * v);
    const float wf[8] = {bf16lo(wr.x), bf16hi(wr.x), bf16lo(wr.y), bf16hi(wr.y),
                         bf16lo(wr.z), bf16hi(wr.z), bf16lo(wr.w), bf16hi(wr.w)};
#pragma unroll
    for (int i = 0; i < 8; ++i) n[8 * v + i] = round_bf16(wf[i] * round_bf16(x[8 * v + i] * inv));
  }
  const float4 *cs = reinterpret_cast<const float4 *>(p.rope + static_cast<size_t>(m) * 64);
  float o[128];
#pragma unroll
  for (int d2 = 0; d2 < 32; ++d2) {  // (cos, sin) of angles 2 d2 and 2 d2 + 1
    const float4 t = __ldg(cs + d2);
    const int d = 2 * d2;
    o[d] = fmaf(n[d], t.x, -n[d + 64] * t.y);
    o[d + 64] = fmaf(n[d], t.y, n[d + 64] * t.x);
    o[d + 1] = fmaf(n[d + 1], t.z, -n[d + 65] * t.w);
    o[d + 65] = fmaf(n[d + 1], t.w, n[d + 65] * t.z);
  }
  dst = h < nq ? p.q_out + (static_cast<size_t>(h) * p.Lp + m) * 128
               : p.cache + ((static_cast<size_t>(h - nq) * p.cap) + p.pos0 + m) * 128;
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int v = 0; v < 16; ++v) {
    uint4 wv;
    wv.x = pack_bf16x2(o[8 * v + 0], o[8 * v + 1]);
    wv.y = pack_bf16x2(o[8 * v + 2], o[8 * v + 3]);
    wv.z = pack_bf16x2(o[8 * v + 4], o[8 * v + 5]);
    wv.w = pack_bf16x2(o[8 * v + 6], o[8 * v + 7]);
    d4[v] = wv;
  }
}

// ---------------------------------------------------------------- kernel
template <class S>
__device__ __forceinline__ bool warp_wait(S &s, uint64_t *bar, uint32_t parity) {
  bool ok = !aborted(s) && mbar_wait(bar, parity);
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) set_abort(s);
  return ok;
}

template <int BN, int MH>
__global__ void __launch_bounds__(NTHREADS, 1) gemm_kernel(const __grid_constant__ Params p) {
  using C = Cfg<BN, MH>;
  using S = Smem<BN, MH>;
  extern __shared__ uint8_t smem_raw[];
  S &s = *reinterpret_cast<S *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int TM = BM * MH;  // rows per tile
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kblocks = p.K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s.acc_full[b], 1);
      mbar_init(&s.acc_empty[b], kEpiThreads);
    }
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tm_a);
    prefetch_tmap(&p.tm_b);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  pdl_launch_dependents();
  pdl_wait();  // A is the previous kernel's output; C may still be read by it

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
        const int m0 = (tile % p.num_m) * TM, nb = tile / p.num_m;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int st = it % C::NS;
          if (it >= C::NS && (aborted(s) || !mbar_wait(&s.empty[st], ((it / C::NS) - 1) & 1))) {
            set_abort(s);
            ok = false;
            break;
          }
          uint8_t *a = s.stage[st];
          uint8_t *b = a + C::A_BYTES;
          mbar_arrive_expect_tx(&s.full[st], C::STAGE);
          tma_load_2d(a, &p.tm_a, kb * BK, m0, &s.full[st]);
          if (p.epi == kSwiGLU) {  // gate rows f0.., then up rows F + f0..
            tma_load_2d(b, &p.tm_b, kb * BK, nb * (BN / 2), &s.full[st]);
            tma_load_2d(b + C::B_BYTES / 2, &p.tm_b, kb * BK, p.swiglu_f + nb * (BN / 2), &s.full[st]);
          } else {
            tma_load_2d(b, &p.tm_b, kb * BK, nb * BN, &s.full[st]);
          }
        }
      }
      // drain: every copy issued must land before the CTA may exit
      for (int t = max(0, it - C::NS); t < it; ++t) mbar_wait(&s.full[t % C::NS], (t / C::NS) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++lt) {
        const int buf = lt % C::NBUF;
        if (lt >= C::NBUF && (aborted(s) || !mbar_wait(&s.acc_empty[buf], ((lt / C::NBUF) - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * MH * BN;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int st = it % C::NS;
          if (aborted(s) || !mbar_wait(&s.full[st], (it / C::NS) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(s.stage[st]);
          const uint32_t b = a + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
#pragma unroll
            for (int h = 0; h < MH; ++h)  // the halves share the W stage
              tc_mma_ss(d + h * BN, sw128_desc(a + h * C::A_HALF + kk * 32), sw128_desc(b + kk * 32), C::IDESC,
                        (kb | kk) != 0);
          tc_commit(&s.empty[st]);
        }
        if (!ok) break;
        tc_commit(&s.acc_full[buf]);
      }
      if (!ok) set_abort(s);
      tc_commit(&s.mma_done);
      mbar_wait(&s.mma_done, 0);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int lt = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
      const int buf = lt % C::NBUF;
      if (!warp_wait(s, &s.acc_full[buf], (lt / C::NBUF) & 1)) break;
      tc_fence_after();
      const int nb = tile / p.num_m;
#pragma unroll 1
      for (int h = 0; h < MH; ++h) {
        const int m = (tile % p.num_m) * TM + h * BM + row;
        const uint32_t ta = tmem + (static_cast<uint32_t>(quad * 32) << 16) + (buf * MH + h) * BN;
        if (p.epi == kSwiGLU) {
          if constexpr (BN == 256) epi_swiglu(p, ta, m, nb * 128);
        } else if (p.epi == kQKRope) {
#pragma unroll 1
          for (int hh = 0; hh < BN / 128; ++hh) epi_qk_rope(p, ta + 128 * hh, m, nb * (BN / 128) + hh);
        } else {
          if (p.epi == kF32Owner)
            epi_store_owner<BN>(p, ta, m - lane, nb * BN, s.ostage[quad]);
          else
            epi_store<BN>(p, ta, m, nb * BN);
        }
      }
      tc_fence_before();
      mbar_arrive(&s.acc_empty[buf]);
    }
    // Partials stored to other GPUs are visible system-wide before the
    // kernel ends; the exchange's next kernel publishes them with a flag.
    if (p.epi == kF32Owner) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---------------------------------------------------------------- few rows
// C = epi(X W^T) for X of M <= 64 rows (a batched decode step, a short
// prompt): the weights are the operand that has to stream, so the roles swap
// (the tcgen05 tile is 128 weight rows x 64 tokens, D^T = W X^T) and K is
// split so that the launch fills the GPU: CTA (r, s) multiplies weight rows
// [128 r, 128 r + 128) by X over k-blocks [s kps, (s + 1) kps) and stores
// its FP32 partial [128][64] to part[s]; gemm_small_reduce_kernel then sums
// the partials of each output in split order (deterministic) and applies the
// epilogue.  Every weight byte is read once; the weight k-blocks of the
// first stages are requested before the programmatic-launch wait (model
// constants), X's after it.
constexpr int kSmallTok = 64;  // token rows per tile (MMA N), X rows >= M zero-filled by TMA
constexpr int kSmallNS = 4;    // pipeline stages
constexpr uint32_t kSmallIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                 (static_cast<uint32_t>(kSmallTok >> 3) << 17) |
                                 (static_cast<uint32_t>(BM >> 4) << 24);
constexpr int kSmallWBytes = BM * BK * 2;         // 16 KB
constexpr int kSmallXBytes = kSmallTok * BK * 2;  // 8 KB

struct SmallParams {
  CUtensorMap tm_w;  // W [N][K], box (64, 128)
  CUtensorMap tm_x;  // X [M][K], box (64, 64)
  int M, N, K;
  int kps;           // k-blocks per split
  float *part;       // [splits][N][64] FP32 partials
};

struct SmallSmem {
  alignas(1024) uint8_t w[kSmallNS][kSmallWBytes];
  alignas(1024) uint8_t x[kSmallNS][kSmallXBytes];
  uint64_t full[kSmallNS], empty[kSmallNS];
  uint64_t acc_full, mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

__global__ void __launch_bounds__(NTHREADS, 2) gemm_small_kernel(const __grid_constant__ SmallParams p) {
  extern __shared__ uint8_t smem_raw[];
  SmallSmem &s = *reinterpret_cast<SmallSmem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int kb0 = split * p.kps, nkb = min(p.K / BK, kb0 + p.kps) - kb0;  // >= 1 (host)

  if (threadIdx.x == 0) {
    for (int i = 0; i < kSmallNS; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.acc_full, 1);
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tm_w);
    prefetch_tmap(&p.tm_x);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kSmallTok);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const int pre = min(nkb, kSmallNS);
      for (int i = 0; i < pre; ++i) {  // weights: no dependence on the previous kernel
        mbar_arrive_expect_tx(&s.full[i], kSmallWBytes + kSmallXBytes);
        tma_load_2d(s.w[i], &p.tm_w, (kb0 + i) * BK, tile * BM, &s.full[i]);
      }
      pdl_wait();  // X is the previous kernel's output
      for (int i = 0; i < pre; ++i) tma_load_2d(s.x[i], &p.tm_x, (kb0 + i) * BK, 0, &s.full[i]);
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const int st = i % kSmallNS;
        if (aborted(s) || !mbar_wait(&s.empty[st], ((i / kSmallNS) - 1) & 1)) {
          set_abort(s);
          break;
        }
        mbar_arrive_expect_tx(&s.full[st], kSmallWBytes + kSmallXBytes);
        tma_load_2d(s.w[st], &p.tm_w, (kb0 + i) * BK, tile * BM, &s.full[st]);
        tma_load_2d(s.x[st], &p.tm_x, (kb0 + i) * BK, 0, &s.full[st]);
        issued = i + 1;
      }
      // drain: every copy issued must land before the CTA may exit
      for (int t = max(0, issued - kSmallNS); t < issued; ++t) mbar_wait(&s.full[t % kSmallNS], (t / kSmallNS) & 1);
    } else {
      pdl_wait();
    }
    __syncwarp();
  } else if (warp == 1) {
    pdl_wait();
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int st = i % kSmallNS;
        if (aborted(s) || !mbar_wait(&s.full[st], (i / kSmallNS) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(s.w[st]), b = smem_u32(s.x[st]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_ss(tmem, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), kSmallIdesc, (i | kk) != 0);
        tc_commit(&s.empty[st]);
      }
      if (ok) tc_commit(&s.acc_full);
      else set_abort(s);
      tc_commit(&s.mma_done);
      mbar_wait(&s.mma_done, 0);
    }
    __syncwarp();
  } else {
    pdl_wait();  // the partials may still be read by the previous call's reduction
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    const int n = tile * BM + quad * 32 + lane;  // weight row = output column
    if (warp_wait(s, &s.acc_full, 0)) {
      tc_fence_after();
      uint32_t r0[32], r1[32];
      const uint32_t ta = tmem + (static_cast<uint32_t>(quad * 32) << 16);
      tmem_ld32(ta, r0);
      tmem_ld32(ta + 32, r1);
      tmem_wait_ld();
      float4 *dst = reinterpret_cast<float4 *>(p.part + (static_cast<size_t>(split) * p.N + n) * kSmallTok);
#pragma unroll
      for (int v = 0; v < 8; ++v)
        dst[v] = make_float4(__uint_as_float(r0[4 * v]), __uint_as_float(r0[4 * v + 1]),
                             __uint_as_float(r0[4 * v + 2]), __uint_as_float(r0[4 * v + 3]));
#pragma unroll
      for (int v = 0; v < 8; ++v)
        dst[8 + v] = make_float4(__uint_as_float(r1[4 * v]), __uint_as_float(r1[4 * v + 1]),
                                 __uint_as_float(r1[4 * v + 2]), __uint_as_float(r1[4 * v + 3]));
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kSmallTok);
}

struct SmallReduceParams {
  const float *part;  // [splits][N][64]
  int splits, N, M;
  int swiglu_f;       // > 0: SwiGLU over gate rows [0, F) and up rows [F, 2F)
  uint16_t *c;        // BF16 [M][ldc]
  long long ldc;
};

// Sums the partials of 8 output columns x 64 tokens in split order
// (thread = token m and columns c, c + 4; the loads of 8 splits are in
// flight at once), applies the epilogue (BF16 store, or SwiGLU with the
// rounding points of epi_swiglu) and writes the M valid token rows, 16 bytes
// per row.
constexpr int kReduceCols = 8;
__global__ void __launch_bounds__(256) gemm_small_reduce_kernel(const __grid_constant__ SmallReduceParams p) {
  __shared__ float t[kSmallTok][kReduceCols + 1];
  pdl_launch_dependents();
  pdl_wait();
  const int n0 = blockIdx.x * kReduceCols;
  const int m = threadIdx.x & 63, c = threadIdx.x >> 6;
  const size_t ss = static_cast<size_t>(p.N) * kSmallTok;  // split stride
  const int nsrc = p.swiglu_f > 0 ? 4 : 2;
  const float *src[4];
  src[0] = p.part + static_cast<size_t>(n0 + c) * kSmallTok + m;
  src[1] = src[0] + 4 * kSmallTok;
  src[2] = src[0] + static_cast<size_t>(p.swiglu_f) * kSmallTok;  // up rows (SwiGLU)
  src[3] = src[2] + 4 * kSmallTok;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s0 = 0; s0 < p.splits; s0 += 8) {
    float v[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int u = 0; u < 8; ++u) v[k][u] = (k < nsrc && s0 + u < p.splits) ? __ldcg(src[k] + (s0 + u) * ss) : 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < p.splits) acc[k] += v[k][u];
  }
  if (p.swiglu_f > 0) {
    acc[0] = silu_bf16(round_bf16(acc[0])) * round_bf16(acc[2]);
    acc[1] = silu_bf16(round_bf16(acc[1])) * round_bf16(acc[3]);
  }
  t[m][c] = acc[0];
  t[m][c + 4] = acc[1];
  __syncthreads();
  if (threadIdx.x < p.M) {
    const float *r = t[threadIdx.x];
    uint4 w;
    w.x = pack_bf16x2(r[0], r[1]);
    w.y = pack_bf16x2(r[2], r[3]);
    w.z = pack_bf16x2(r[4], r[5]);
    w.w = pack_bf16x2(r[6], r[7]);
    *reinterpret_cast<uint4 *>(p.c + static_cast<size_t>(threadIdx.x) * p.ldc + n0) = w;
  }
}

// ---------------------------------------------------------------- RoPE table
// (cos, sin) of the 64 angles of positions pos0 .. pos0 + count - 1, each as
// rope::rope_angles forms it; one CTA of 64 threads per position.
__global__ void rope_table_kernel(int pos0, int count, const __grid_constant__ rope::Params rp, float2 *table) {
  __shared__ float c[64], sn[64];
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x;
  rope::rope_angles(pos0 + i, rp.inv_freq, c, sn, threadIdx.x);
  __syncthreads();
  if (threadIdx.x < 64) table[static_cast<size_t>(i) * 64 + threadIdx.x] = make_float2(c[threadIdx.x], sn[threadIdx.x]);
}

}  // namespace gemm
}  // namespace rib
