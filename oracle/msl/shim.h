// Metal Shading Language built-ins for running the reference's Metal compute
// kernels on the CPU -- TEST INFRASTRUCTURE ONLY.
//
// The reference (aeilot/roofline-inference, agent-test/v2/kernels.py and
// attention.py) holds its hot-path kernels as MSL source strings that
// mx.fast.metal_kernel compiles.  oracle/msl/runner.py captures those exact
// strings and launch shapes from the reference's own Python host code and
// compiles each body as C++ against this header, so the oracle can be checked
// against the reference's kernels, not only against a restatement of them.
//
// Execution model.  A threadgroup's threads run as cooperative fibers on one
// host thread, scheduled round robin.  Every cross-thread operation (SIMD-group
// reductions and shuffles, SIMD-group matrix products, threadgroup barriers)
// is a scheduling point: a thread deposits its operand, yields until every
// other thread of the threadgroup has reached its own next scheduling point,
// reads the combined result and yields once more, so no deposit is overwritten
// before every lane has read it.  This is the hardware's lock-step semantics
// for kernels whose SIMD groups take uniform control flow, which each
// collective checks (all 32 lanes must arrive, in the same collective).
//
// Stand-ins that cannot match Apple's hardware bit for bit:
//   - metal::fast::{cos, sin, exp2} and metal::{exp, exp2}: the C library's
//     correctly rounded (or nearly so) float functions;
//   - simd_sum: the xor-butterfly order (offsets 16, 8, 4, 2, 1);
//   - simdgroup_multiply_accumulate: FP32 products and sums in k order;
//   - dot(float4, float4): ((x0 y0 + x1 y1) + x2 y2) + x3 y3, no fused multiply-add.
// threadgroup storage is a thread_local static (one threadgroup runs at a time
// per host thread).
#pragma once

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <ucontext.h>

#include <algorithm>
#include <cmath>

#define device
#define constant
#define TG_STATIC static thread_local

typedef unsigned int uint;
typedef unsigned short ushort;
typedef uint64_t ulong;

struct uint3 {
  uint x, y, z;
};
struct uint4 {
  uint x, y, z, w;
};
struct ulong2 {
  ulong x, y;
  ulong2(ulong a = 0, ulong b = 0) : x(a), y(b) {}
};

// ------------------------------------------------------------------ bfloat16
struct bfloat16_t {
  uint16_t bits;
  bfloat16_t() : bits(0) {}
  explicit bfloat16_t(float f) {  // round to nearest even
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {
      bits = static_cast<uint16_t>((u >> 16) | ((u & 0xffffu) ? 0x40u : 0u));
    } else {
      u += 0x7fffu + ((u >> 16) & 1u);
      bits = static_cast<uint16_t>(u >> 16);
    }
  }
  explicit bfloat16_t(double d) : bfloat16_t(static_cast<float>(d)) {}
  explicit bfloat16_t(int i) : bfloat16_t(static_cast<float>(i)) {}
  operator float() const {
    uint32_t u = static_cast<uint32_t>(bits) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
};

// ------------------------------------------------------------------ vectors
struct float4 {
  float x, y, z, w;
  float4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
};
struct ushort4 {
  ushort x, y, z, w;
};
typedef ushort4 packed_ushort4;
struct bfloat4 {
  bfloat16_t x, y, z, w;
  operator float4() const { return float4(float(x), float(y), float(z), float(w)); }
};
template <typename T, typename S>
inline T as_type(const S &s) {
  static_assert(sizeof(T) == sizeof(S), "as_type size");
  T t;
  memcpy(&t, &s, sizeof(T));
  return t;
}
inline float dot(const float4 &a, const float4 &b) {
  float p0 = a.x * b.x, p1 = a.y * b.y, p2 = a.z * b.z, p3 = a.w * b.w;
  return ((p0 + p1) + p2) + p3;
}

namespace metal {
template <typename T>
inline T max(T a, T b) { return a > b ? a : b; }
template <typename T>
inline T min(T a, T b) { return a < b ? a : b; }
inline float exp2(float x) { return ::exp2f(x); }
inline float exp(float x) { return ::expf(x); }
namespace precise {
inline float rsqrt(float x) { return static_cast<float>(1.0 / ::sqrt(static_cast<double>(x))); }
}  // namespace precise
namespace fast {
inline float cos(float x) { return ::cosf(x); }
inline float sin(float x) { return ::sinf(x); }
inline float exp2(float x) { return ::exp2f(x); }
}  // namespace fast
}  // namespace metal
namespace fast = metal::fast;
using metal::max;
using metal::min;

// ------------------------------------------------------------------ fibers
namespace msl {

constexpr int kMaxThreads = 1024;
constexpr size_t kStack = 256 * 1024;

struct Fiber {
  ucontext_t ctx;
  bool alive;
  int tid;
};

struct Group {  // per host thread: the threadgroup being run
  Fiber fib[kMaxThreads];
  ucontext_t sched;
  int n;
  int cur;
  // per SIMD group deposits (up to 32 SIMD groups of 32 lanes)
  float dep[kMaxThreads][3][2];  // [thread][operand][element]
  float dep1[kMaxThreads];
  unsigned seq[kMaxThreads];     // collectives entered by each thread
  unsigned done[kMaxThreads];    // collectives whose result each thread has read
  int barrier_arrivals;
  unsigned barrier_seq[kMaxThreads];
  char *stacks;
  void (*body)(void *, int);
  void *arg;
};

inline Group &group() {
  static thread_local Group *g = nullptr;
  if (!g) {
    g = static_cast<Group *>(calloc(1, sizeof(Group)));
    g->stacks = static_cast<char *>(malloc(kStack * kMaxThreads));
  }
  return *g;
}

inline void fail(const char *what) {
  fprintf(stderr, "msl shim: %s\n", what);
  abort();
}

inline void yield() {
  Group &g = group();
  swapcontext(&g.fib[g.cur].ctx, &g.sched);
}

inline int self() { return group().cur; }

// A collective of the SIMD group: every lane deposits, all lanes of the group
// must be in the same collective.
inline int lane_base() { return self() & ~31; }

// Yields until every lane of the caller's SIMD group has arr[lane] >= target.
inline void wait_lanes(const unsigned *arr, unsigned target) {
  Group &g = group();
  const int b = lane_base();
  for (;;) {
    bool ok = true;
    for (int l = 0; l < 32; ++l) {
      if (b + l >= g.n) fail("SIMD group extends past the threadgroup");
      if (arr[b + l] >= target) continue;
      if (!g.fib[b + l].alive) fail("SIMD-group collective with an exited lane");
      ok = false;
    }
    if (ok) return;
    yield();
  }
}
// Collective protocol: enter() after depositing, leave() after reading.
inline void simd_enter() {
  Group &g = group();
  const unsigned s = ++g.seq[g.cur];
  wait_lanes(g.seq, s);
  const int b = lane_base();
  for (int l = 0; l < 32; ++l)
    if (g.seq[b + l] != s) fail("SIMD-group collective reached with non-uniform control flow");
}
inline void simd_leave() {
  Group &g = group();
  g.done[g.cur] = g.seq[g.cur];
  wait_lanes(g.done, g.seq[g.cur]);
}

inline void entry(unsigned lo, unsigned hi) {
  (void)lo;
  (void)hi;
  Group &g = group();
  const int t = g.cur;
  g.body(g.arg, t);
  g.fib[t].alive = false;
}

// Runs body(arg, t) for t in [0, n) as one threadgroup.
inline void run_group(int n, void (*body)(void *, int), void *arg) {
  Group &g = group();
  if (n > kMaxThreads || n % 32) fail("threadgroup size must be a multiple of 32, at most 1024");
  g.n = n;
  g.body = body;
  g.arg = arg;
  g.barrier_arrivals = 0;
  for (int t = 0; t < n; ++t) {
    Fiber &f = g.fib[t];
    f.alive = true;
    f.tid = t;
    g.seq[t] = 0;
    g.done[t] = 0;
    g.barrier_seq[t] = 0;
    getcontext(&f.ctx);
    f.ctx.uc_stack.ss_sp = g.stacks + kStack * t;
    f.ctx.uc_stack.ss_size = kStack;
    f.ctx.uc_link = &g.sched;
    makecontext(&f.ctx, reinterpret_cast<void (*)()>(entry), 2, 0u, 0u);
  }
  for (;;) {
    bool any = false;
    for (int t = 0; t < n; ++t) {
      if (!g.fib[t].alive) continue;
      any = true;
      g.cur = t;
      swapcontext(&g.sched, &g.fib[t].ctx);
    }
    if (!any) break;
  }
}

}  // namespace msl

// ------------------------------------------------------------------ SIMD-group functions
inline float simd_sum(float v) {
  msl::Group &g = msl::group();
  const int me = g.cur;
  g.dep1[me] = v;
  msl::simd_enter();
  const int b = msl::lane_base();
  float s[32];
  for (int l = 0; l < 32; ++l) s[l] = g.dep1[b + l];
  for (int off = 16; off >= 1; off >>= 1) {
    float t[32];
    for (int l = 0; l < 32; ++l) t[l] = s[l] + s[l ^ off];
    memcpy(s, t, sizeof(s));
  }
  const float r = s[me - b];
  msl::simd_leave();
  return r;
}

inline float simd_shuffle_xor(float v, ushort mask) {
  msl::Group &g = msl::group();
  const int me = g.cur;
  g.dep1[me] = v;
  msl::simd_enter();
  const int b = msl::lane_base();
  const float r = g.dep1[b + (((me - b) ^ mask) & 31)];
  msl::simd_leave();
  return r;
}

inline bool simd_all(bool v) {
  msl::Group &g = msl::group();
  const int me = g.cur;
  g.dep1[me] = v ? 1.f : 0.f;
  msl::simd_enter();
  const int b = msl::lane_base();
  bool r = true;
  for (int l = 0; l < 32; ++l) r = r && g.dep1[b + l] != 0.f;
  msl::simd_leave();
  return r;
}

namespace mem_flags {
constexpr int mem_threadgroup = 1;
constexpr int mem_device = 2;
}  // namespace mem_flags

// Every thread of the threadgroup that has not exited must arrive.
inline void threadgroup_barrier(int) {
  msl::Group &g = msl::group();
  const unsigned s = ++g.barrier_seq[g.cur];
  for (;;) {
    bool ok = true;
    for (int t = 0; t < g.n; ++t) ok = ok && (!g.fib[t].alive || g.barrier_seq[t] >= s);
    if (ok) return;
    msl::yield();
  }
}

// ------------------------------------------------------------------ SIMD-group matrices
// An 8x8 matrix spread over the 32 lanes: lane l holds row fm, columns fn and
// fn + 1, with q = l / 4, fm = (q & 4) + (l / 2) % 4, fn = (q & 2) * 2 + (l % 2) * 2
// -- the layout the reference kernel itself assumes (attention.py:46-48).
inline void frag_pos(int lane, int &fm, int &fn) {
  const int q = lane / 4;
  fm = (q & 4) + ((lane / 2) % 4);
  fn = (q & 2) * 2 + (lane % 2) * 2;
}

template <typename T, int C, int R>
struct simdgroup_matrix {
  static_assert(C == 8 && R == 8, "8x8 only");
  T e[2];
  simdgroup_matrix() : e{T(0.0f), T(0.0f)} {}
  explicit simdgroup_matrix(T dval) {  // dval on the diagonal, zero elsewhere
    int fm, fn;
    frag_pos(msl::self() & 31, fm, fn);
    e[0] = (fm == fn) ? dval : T(0.0f);
    e[1] = (fm == fn + 1) ? dval : T(0.0f);
  }
  T *thread_elements() { return e; }
};

template <typename T, typename S>
inline void simdgroup_load(simdgroup_matrix<T, 8, 8> &m, const S *src, ulong elements_per_row,
                           ulong2 origin = ulong2(0, 0), bool transpose = false) {
  int fm, fn;
  frag_pos(msl::self() & 31, fm, fn);
  for (int j = 0; j < 2; ++j) {
    const ulong r = fm, c = fn + j;
    const S v = transpose ? src[(origin.y + c) * elements_per_row + origin.x + r]
                          : src[(origin.y + r) * elements_per_row + origin.x + c];
    m.e[j] = T(float(v));
  }
}

template <typename TD, typename TA, typename TB, typename TC>
inline void simdgroup_multiply_accumulate(simdgroup_matrix<TD, 8, 8> &d, const simdgroup_matrix<TA, 8, 8> &a,
                                          const simdgroup_matrix<TB, 8, 8> &b,
                                          const simdgroup_matrix<TC, 8, 8> &c) {
  msl::Group &g = msl::group();
  const int me = g.cur;
  for (int j = 0; j < 2; ++j) {
    g.dep[me][0][j] = float(a.e[j]);
    g.dep[me][1][j] = float(b.e[j]);
    g.dep[me][2][j] = float(c.e[j]);
  }
  msl::simd_enter();
  const int base = msl::lane_base();
  float A[8][8], B[8][8];
  for (int l = 0; l < 32; ++l) {
    int fm, fn;
    frag_pos(l, fm, fn);
    for (int j = 0; j < 2; ++j) {
      A[fm][fn + j] = g.dep[base + l][0][j];
      B[fm][fn + j] = g.dep[base + l][1][j];
    }
  }
  int fm, fn;
  frag_pos(me - base, fm, fn);
  float out[2];
  for (int j = 0; j < 2; ++j) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += A[fm][k] * B[k][fn + j];
    out[j] = g.dep[me][2][j] + s;
  }
  msl::simd_leave();
  d.e[0] = TD(out[0]);
  d.e[1] = TD(out[1]);
}
