// Causal GQA flash attention for prefill on sm_100a: tcgen05.mma with TMEM
// accumulators, operands staged by TMA.
//
// Replaces the Metal kernel attention() of agent-test/v2/attention.py:18-185:
// same layouts (Q [H, qLp, 128], K/V cache halves [nkv, cap, 128], O
// [qL, H*128]), GQA pairing (both query heads of a KV head in one CTA,
// attention.py:3-5), bottom-right aligned causal mask (query i sees keys
// <= kL - qL + i, attention.py:24,111), online softmax in the exp2 domain
// (attention.py:59), whole masked key tiles skipped (attention.py:87) and
// heavy query blocks scheduled first (attention.py:26).
//
// CTA = 128 query rows x one KV head g (query heads 2g, 2g+1), 12 warps in
// three warpgroups:
//   warp 0      TMA producer: Q of both heads once, then K and V tiles of
//               128 keys into 2-stage rings (128B-swizzled panels).
//   warp 1      TMEM owner and MMA issuer (one thread):
//                 S_h = Q_h K^T       SS-MMA, M=N=128, K=128 (8 x K16)
//                 O_h += P_h V        TS-MMA, A = P_h from TMEM, B = V (MN-major)
//               issue order PV_0(j), S_0(j+1), PV_1(j), S_1(j+1), so the tensor
//               pipe works on one head while the other head's softmax runs.
//   warps 2-3   idle (they complete the first warpgroup for the register split)
// P.V runs as an FP16 MMA on FP16 P: P carries 11 significant bits instead of
// BF16's 8, and the output error stays at the BF16 rounding floor, the
// accuracy of the reference kernel's FP32 P (attention.py:6, 141-153).  A
// kind::f16 MMA takes A and B of one type, so V is read from an FP16 copy
// that v_half_kernel writes once per call (exact for |v| <= 65504; larger
// values are flagged on the device status word as RIB_EINVAL): 2 bytes per
// key and head each way, about 0.5% of a 32k prefill's time.
//   warps 4-7   softmax of head 2g   (one thread per query row / TMEM lane)
//   warps 8-11  softmax of head 2g+1
// Registers: launched at 168 per thread; warpgroup 0 gives back to 40
// (setmaxnreg.dec) and the softmax warpgroups take 232 (setmaxnreg.inc), so a
// softmax thread holds its whole 128-column score row after one TMEM read.
// Per SM sub-partition that is 40 + 232 + 232 = 504 <= 512 registers per
// lane, and 128*40 + 256*232 = 384*168, the launch allocation exactly; the
// host refuses to launch unless the kernel really was built at 168.
// TMEM (512 columns): S_0 [0,128), S_1 [128,256) as FP32; P_h is written as
// packed FP16 over the first 64 columns of S_h; O_0 [256,384), O_1 [384,512).
// The running max is only raised (and O rescaled) when it grows by more
// than 8 in log2 units; until then exp2 arguments stay below 8 and P below
// 256, well inside FP16's range, with 11 significant bits.
// Every wait is bounded (common.cuh); on a timeout the CTA sets a flag,
// drains, frees TMEM and returns.
#pragma once

#include <cuda.h>

#include <algorithm>

#include "common.cuh"

namespace rib {
namespace prefill {

constexpr int D = 128;
constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // keys per tile
constexpr int NS = 2;    // K pipeline stages
constexpr int NSV = 2;   // V pipeline stages
constexpr int NWARPS = 12;
constexpr int NTHREADS = NWARPS * 32;
constexpr int PANEL_BYTES = 128 * 128;          // [128 rows][64 dims] BF16, one swizzle panel
constexpr int TILE_BYTES = 2 * PANEL_BYTES;     // [128 rows][128 dims]
constexpr uint32_t TMEM_COLS = 512;
#ifndef RIB_PREFILL_RESCALE_LOG2
#define RIB_PREFILL_RESCALE_LOG2 8.0f
#endif
constexpr float kRescaleThreshold = RIB_PREFILL_RESCALE_LOG2;  // log2 units
constexpr int kLaunchRegs = 168;                 // registers per thread at launch
constexpr int kRegsLow = 40;                     // warpgroup 0 after setmaxnreg.dec
constexpr int kRegsHigh = 232;                   // softmax warpgroups after setmaxnreg.inc
static_assert(128 * kRegsLow + 256 * kRegsHigh <= NTHREADS * kLaunchRegs,
              "register split exceeds the launch allocation");
static_assert(kRegsLow + 2 * kRegsHigh <= 512, "register split exceeds one sub-partition");

// Instruction descriptor, kind::f16: D = F32 (bits 4-5 = 1), A = B = BF16
// (bits 7-9, 10-12 = 1), N >> 3 at bits 17-22, M >> 4 at bits 24-28;
// bit 16 = B is MN-major.
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) |
                                (static_cast<uint32_t>(BN >> 3) << 17) |
                                (static_cast<uint32_t>(BM >> 4) << 24);
constexpr uint32_t kIdescS = kIdescBase;              // A, B K-major
// P.V: A = P (TMEM) and B = V (MN-major) both FP16 (format 0 at bits 7-9, 10-12).
constexpr uint32_t kIdescPV = ((kIdescBase & ~((7u << 7) | (7u << 10)))) | (1u << 16);

struct Smem {
  alignas(1024) uint8_t q[2][TILE_BYTES];
  alignas(1024) uint8_t k[NS][TILE_BYTES];
  alignas(1024) uint8_t v[NSV][TILE_BYTES];
  uint64_t q_full;
  uint64_t k_full[NS], k_empty[NS];
  uint64_t v_full[NSV], v_empty[NSV];
  uint64_t s_full[2], p_full[2], o_full[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

struct Params {
  CUtensorMap tm_q;  // (128, qLp, H)   box (64, 128, 1), 128B swizzle
  CUtensorMap tm_k;  // (128, kL, nkv)  row stride 256 B, head stride cap*256 B
  CUtensorMap tm_v;
  uint16_t *out;     // [qL][H*128]
  int qL, kL, H, nkv, off, nqb;
  float scale_log2;
};

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2 at bits
// 61-63), sm100 version bit 46; address, LBO and SBO in 16-byte units.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ bool aborted(const Smem &s) {
  return *reinterpret_cast<const volatile int *>(&s.abort_flag) != 0;
}
__device__ __forceinline__ void set_abort(Smem &s) {
  *reinterpret_cast<volatile int *>(&s.abort_flag) = 1;
}

__device__ __forceinline__ uint64_t pack2f(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ uint64_t pack2u(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
__device__ __forceinline__ void unpack2f(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
// Two FP32 lanes per instruction (sm_100 packed FP32).
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Two BF16 values -> two FP16 values (round to nearest; exact for normal
// magnitudes up to 65504); `bad` collects results that overflowed to inf
// (or NaN inputs).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t w, uint32_t &bad) {
  const uint32_t r = pack_f16x2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  bad |= static_cast<uint32_t>((r & 0x7C00u) == 0x7C00u) | static_cast<uint32_t>((r & 0x7C000000u) == 0x7C000000u);
  return r;
}

// Causal / length mask of 32 score columns starting at key `key0`.
__device__ __forceinline__ void mask_chunk(uint32_t (&r)[32], int key0, int my_last, int kL) {
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const int key = key0 + e;
    if (key > my_last || key >= kL) r[e] = __float_as_uint(-INFINITY);
  }
}

// Warp-uniform bounded wait: every lane waits, then all agree.
__device__ __forceinline__ bool warp_wait(Smem &s, uint64_t *bar, uint32_t parity) {
  bool ok = !aborted(s) && mbar_wait(bar, parity);
  ok = __all_sync(0xffffffffu, ok);
  if (!ok) set_abort(s);
  return ok;
}

__global__ void __launch_bounds__(NTHREADS, 1) prefill_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem &s = *reinterpret_cast<Smem *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int qb = p.nqb - 1 - static_cast<int>(blockIdx.x) / p.nkv;  // heavy blocks first
  const int g = static_cast<int>(blockIdx.x) % p.nkv;
  const int q0 = qb * BM;
  const int q_last = min(q0 + BM - 1, p.qL - 1);
  const int last_key = min(p.kL - 1, p.off + q_last);
  const int nt = last_key / BN + 1;  // key tiles this CTA visits

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&s.s_full[h], 1);
      mbar_init(&s.p_full[h], 128);
      mbar_init(&s.o_full[h], 1);
    }
    mbar_init(&s.mma_done, 1);
    s.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tm_q);
    prefetch_tmap(&p.tm_k);
    prefetch_tmap(&p.tm_v);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp < 4) {
    // warpgroup 0: producer, MMA issuer, two V-converter warps
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&s.q_full, 2 * TILE_BYTES);
      for (int h = 0; h < 2; ++h)
        for (int c = 0; c < 2; ++c)
          tma_load_3d(s.q[h] + c * PANEL_BYTES, &p.tm_q, c * 64, q0, 2 * g + h, &s.q_full);
      // K tiles in a 2-stage ring, V tiles in a 3-stage ring: V runs a tile
      // further ahead, so its FP16 conversion is done before P.V needs it.
      int issued_k = 0, issued_v = 0;
      for (int t = 0; t < nt; ++t) {
        const int sk = t % NS, sv = t % NSV;
        if (t >= NS && (aborted(s) || !mbar_wait(&s.k_empty[sk], ((t / NS) - 1) & 1))) {
          set_abort(s);
          break;
        }
        mbar_arrive_expect_tx(&s.k_full[sk], TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_3d(s.k[sk] + c * PANEL_BYTES, &p.tm_k, c * 64, t * BN, g, &s.k_full[sk]);
        issued_k = t + 1;
        if (t >= NSV && (aborted(s) || !mbar_wait(&s.v_empty[sv], ((t / NSV) - 1) & 1))) {
          set_abort(s);
          break;
        }
        mbar_arrive_expect_tx(&s.v_full[sv], TILE_BYTES);
        for (int c = 0; c < 2; ++c)
          tma_load_3d(s.v[sv] + c * PANEL_BYTES, &p.tm_v, c * 64, t * BN, g, &s.v_full[sv]);
        issued_v = t + 1;
      }
      // drain: every copy issued must land before the CTA may exit
      mbar_wait(&s.q_full, 0);
      for (int t = max(0, issued_k - NS); t < issued_k; ++t) mbar_wait(&s.k_full[t % NS], (t / NS) & 1);
      for (int t = max(0, issued_v - NSV); t < issued_v; ++t) mbar_wait(&s.v_full[t % NSV], (t / NSV) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      auto issue_s = [&](int h, int st) {
        const uint32_t qa = smem_u32(s.q[h]), kb = smem_u32(s.k[st]);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off = (k >> 2) * PANEL_BYTES + (k & 3) * 32;
          tc_mma_ss(tmem + h * 128, sw128_desc(qa + off, 16, 1024), sw128_desc(kb + off, 16, 1024),
                    kIdescS, k > 0);
        }
      };
      auto issue_pv = [&](int h, int st, bool first) {
        const uint32_t vb = smem_u32(s.v[st]);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          tc_mma_ts(tmem + 256 + h * 128, tmem + h * 128 + k * 8,
                    sw128_desc(vb + k * 2048, PANEL_BYTES, 1024), kIdescPV, (!first || k > 0));
      };
      bool ok = mbar_wait(&s.q_full, 0) && mbar_wait(&s.k_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        tc_commit(&s.s_full[0]);
        issue_s(1, 0);
        tc_commit(&s.s_full[1]);
        tc_commit(&s.k_empty[0]);  // K stage free once both S MMAs have run
      }
      for (int j = 0; ok && j < nt; ++j) {
        const int sv = j % NSV, sk1 = (j + 1) % NS;
        ok = !aborted(s) && mbar_wait(&s.v_full[sv], (j / NSV) & 1) &&
             mbar_wait(&s.p_full[0], j & 1);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, sv, j == 0);
        tc_commit(&s.o_full[0]);
        if (j + 1 < nt) {
          if (!(ok = mbar_wait(&s.k_full[sk1], ((j + 1) / NS) & 1))) break;
          tc_fence_after();
          issue_s(0, sk1);
          tc_commit(&s.s_full[0]);
        }
        if (!(ok = !aborted(s) && mbar_wait(&s.p_full[1], j & 1))) break;
        tc_fence_after();
        issue_pv(1, sv, j == 0);
        tc_commit(&s.o_full[1]);
        tc_commit(&s.v_empty[sv]);
        if (j + 1 < nt) {
          issue_s(1, sk1);
          tc_commit(&s.s_full[1]);
          tc_commit(&s.k_empty[sk1]);
        }
      }
      if (!ok) set_abort(s);
      tc_commit(&s.mma_done);
      mbar_wait(&s.mma_done, 0);
    }
    __syncwarp();
  }
  } else {
    // warpgroups 1 and 2: softmax
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax
    const int h = (warp - 4) >> 2;           // 0 for warps 4-7, 1 for warps 8-11
    const int quad = warp & 3;               // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;        // query row within the block
    const int q_row = q0 + row;
    const int my_last = p.off + q_row;       // last visible key (inclusive)
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t tS = lane_base + h * 128;
    const uint32_t tO = lane_base + 256 + h * 128;
    const float sl2 = p.scale_log2;
    const uint64_t sl2x2 = pack2f(sl2, sl2);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (!(ok = warp_wait(s, &s.s_full[h], j & 1))) break;
      tc_fence_after();
      const int k0 = j * BN;
      uint32_t r[BN];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
      tmem_wait_ld();
      if (k0 + BN - 1 > p.off + q0 || k0 + BN > p.kL) {  // tile crosses the diagonal or kL
#pragma unroll
        for (int c = 0; c < 4; ++c)
          mask_chunk(*reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]), k0 + c * 32, my_last, p.kL);
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], __uint_as_float(r[c]));
      const float mt = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2;
      const bool need = mt > m + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float mn = fmaxf(m, mt);
        if (j > 0) {
          const float alpha = fast_exp2(m - mn);
          if (!(ok = warp_wait(s, &s.o_full[h], (j - 1) & 1))) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
          l *= alpha;
        }
        m = mn;
      }
      // P = exp2(S * scale*log2e - m), packed FP16 over S's first 64 columns
      // (the whole row is already in registers).
      const uint64_t nm2 = pack2f(-m, -m);
      uint64_t acc0 = pack2f(0.f, 0.f), acc1 = acc0;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = half * 64 + 2 * e;
          float a, b;
          unpack2f(ffma2(pack2u(r[c], r[c + 1]), sl2x2, nm2), a, b);
          a = fast_exp2(a);
          b = fast_exp2(b);
          if (e & 1) acc1 = fadd2(acc1, pack2f(a, b));
          else acc0 = fadd2(acc0, pack2f(a, b));
          pk[e] = pack_f16x2(a, b);
        }
        tmem_st32(tS + half * 32, pk);
      }
      float s0, s1, s2, s3;
      unpack2f(acc0, s0, s1);
      unpack2f(acc1, s2, s3);
      l += (s0 + s1) + (s2 + s3);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&s.p_full[h]);
    }
    // ---- epilogue: O / l -> BF16, row-major [qL, H*128]
    if (ok && warp_wait(s, &s.o_full[h], (nt - 1) & 1)) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      uint32_t o[D];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tO + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&o[c * 32]));
      tmem_wait_ld();
      if (q_row < p.qL) {
        uint4 *d4 = reinterpret_cast<uint4 *>(p.out + static_cast<size_t>(q_row) * (p.H * D) + (2 * g + h) * D);
#pragma unroll
        for (int v = 0; v < D / 8; ++v) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv_l, __uint_as_float(o[8 * v + 1]) * inv_l);
          w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv_l, __uint_as_float(o[8 * v + 3]) * inv_l);
          w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv_l, __uint_as_float(o[8 * v + 5]) * inv_l);
          w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv_l, __uint_as_float(o[8 * v + 7]) * inv_l);
          d4[v] = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// V [nkv][cap][128] BF16 rows [0, kL) -> v16 [nkv][kL][128] FP16 (round to
// nearest: exact for |v| <= 65504; values past the FP16 range become inf and
// are recorded as RIB_EINVAL on the device status word).
__global__ void __launch_bounds__(256) v_half_kernel(const uint16_t *__restrict__ V, int cap, int kL, int nkv,
                                                     uint16_t *__restrict__ v16) {
  const long long per_head = static_cast<long long>(kL) * (D / 8);
  const long long total = per_head * nkv;
  uint32_t bad = 0;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long h = i / per_head, r = i - h * per_head;  // r: 16-byte chunk within the head
    uint4 w = *reinterpret_cast<const uint4 *>(V + h * cap * D + r * 8);
    w.x = bf16x2_to_f16x2(w.x, bad);
    w.y = bf16x2_to_f16x2(w.y, bad);
    w.z = bf16x2_to_f16x2(w.z, bad);
    w.w = bf16x2_to_f16x2(w.w, bad);
    *reinterpret_cast<uint4 *>(v16 + h * kL * D + r * 8) = w;
  }
  if (bad) atomicExch(&g_device_status, RIB_EINVAL);
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr) {
      cudaGetLastError();
      host_fail(RIB_ECUDA, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)",
                e != cudaSuccess ? static_cast<int>(e) : static_cast<int>(q));
      return nullptr;
    }
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 3-D BF16 map (128, rows, heads), row stride 256 B, head stride
// head_stride_rows*256 B; box (64, 128, 1); rows past `rows` read as zero.
inline bool make_map(CUtensorMap *m, const void *base, int rows, int heads, long long head_stride_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(heads)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2),
                           static_cast<cuuint64_t>(head_stride_rows) * D * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims, strides,
                         box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    host_fail(RIB_ECUDA, "cuTensorMapEncodeTiled", static_cast<int>(r));
    return false;
  }
  return true;
}

inline bool g_smem_done[64];

// Bytes of the FP16 copy of V a prefill call needs: [nkv][kL][128].
inline size_t workspace_bytes(int kL, int nkv) {
  return (static_cast<size_t>(nkv) * kL * D * 2 + 255) / 256 * 256;
}

inline int launch(const void *Q, const void *K, const void *V, int qL, int kL, int qLp, int cap,
                  int H, int nkv, float scale, void *O, void *workspace, size_t workspace_bytes_,
                  void *stream, bool (*bind)(void *)) {
  if (!Q || !K || !V || !O || !workspace) return RIB_EINVAL;
  if (nkv < 1 || H != 2 * nkv || qL < 1 || qLp < qL || kL < qL || cap < 1 || !(scale > 0.f))
    return RIB_EINVAL;
  if (kL > cap) return RIB_ECAPACITY;
  if (workspace_bytes_ < workspace_bytes(kL, nkv)) return RIB_EINVAL;
  auto a16 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
  if (!a16(Q) || !a16(K) || !a16(V) || !a16(O) || !a16(workspace)) return RIB_EALIGN;
  if (!bind(stream)) return host_fail(RIB_ECUDA, "bind stream device", 0);
  // V -> FP16 copy [nkv][kL][128]
  uint16_t *v16 = static_cast<uint16_t *>(workspace);
  {
    const long long chunks = static_cast<long long>(nkv) * kL * (D / 8);
    const int threads = 256;
    const int blocks = static_cast<int>(std::min<long long>((chunks + threads - 1) / threads, 148LL * 16));
    v_half_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t *>(V), cap, kL, nkv, v16);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return host_fail_cuda("v_half_kernel launch", e);
  }
  Params p;
  if (!make_map(&p.tm_q, Q, qLp, H, qLp) || !make_map(&p.tm_k, K, kL, nkv, cap) ||
      !make_map(&p.tm_v, v16, kL, nkv, kL))
    return RIB_ECUDA;
  p.out = static_cast<uint16_t *>(O);
  p.qL = qL;
  p.kL = kL;
  p.H = H;
  p.nkv = nkv;
  p.off = kL - qL;
  p.nqb = (qL + BM - 1) / BM;
  p.scale_log2 = scale * 1.4426950408889634f;
  const int smem = static_cast<int>(sizeof(Smem)) + 1024;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return host_fail_cuda("cudaGetDevice", e);
  if (!g_smem_done[dev]) {
    e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return host_fail_cuda("cudaFuncSetAttribute(prefill smem)", e);
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, prefill_kernel);
    if (e != cudaSuccess) return host_fail_cuda("cudaFuncGetAttributes(prefill)", e);
    if (fa.numRegs != kLaunchRegs || fa.maxThreadsPerBlock < NTHREADS ||
        fa.maxDynamicSharedSizeBytes < smem) {
      snprintf(g_last_error, sizeof(g_last_error),
               "prefill_kernel not launched: %d registers/thread (register split needs exactly %d), "
               "max %d threads/block (need %d), max dynamic smem %d (need %d)",
               fa.numRegs, kLaunchRegs, fa.maxThreadsPerBlock, NTHREADS,
               fa.maxDynamicSharedSizeBytes, smem);
      return RIB_ECUDA;
    }
    g_smem_done[dev] = true;
  }
  prefill_kernel<<<p.nqb * nkv, NTHREADS, smem, static_cast<cudaStream_t>(stream)>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa;
    cudaFuncGetAttributes(&fa, prefill_kernel);
    snprintf(g_last_error, sizeof(g_last_error),
             "prefill_kernel launch failed: %s (regs/thread %d, max threads/block %d, smem %d, "
             "max dyn smem %d)", cudaGetErrorName(e), fa.numRegs, fa.maxThreadsPerBlock, smem,
             fa.maxDynamicSharedSizeBytes);
    return RIB_ECUDA;
  }
  return RIB_OK;
}

}  // namespace prefill
}  // namespace rib
