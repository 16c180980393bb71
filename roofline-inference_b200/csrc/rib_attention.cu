// C ABI of the B200 attention hot path: host-side argument checks, launch
// geometry and workspace layout for the kernels in the *.cuh files.
// Built as one translation unit so that all kernels share the device status
// word (common.cuh).
#include <cmath>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "decode_attention.cuh"
#include "decode_step.cuh"
#include "prefill_attention.cuh"
#include "decode_streamk.cuh"
#include "gemm.cuh"
#include "model_kernels.cuh"
#include "qk_norm_rope.cuh"
#include "tp_prefill.cuh"

// Largest split of the decode kernel, in keys (a build-time tuning constant).
#ifndef RIB_DECODE_MAX_CHUNK
#define RIB_DECODE_MAX_CHUNK 4096
#endif
// Fewest waves of decode CTAs a launch is split into (a build-time tuning constant).
#ifndef RIB_DECODE_MIN_WAVES
#define RIB_DECODE_MIN_WAVES 1
#endif
// Decode CTAs per SM that one wave of splits aims to fill (a build-time tuning constant).
#ifndef RIB_DECODE_SLOTS_PER_SM
#define RIB_DECODE_SLOTS_PER_SM 2
#endif
// Decode kernel choice: 0 the fixed-split kernel always, 1 the stream-K
// kernel (decode_streamk.cuh) where use_streamk() finds it faster, 2 stream-K
// for every launch of at most kStreamMaxSeqs sequences.
#ifndef RIB_DECODE_STREAMK
#define RIB_DECODE_STREAMK 1
#endif

namespace {

constexpr int kMaxDevices = 64;

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return dev;
}

// SM count of the current device (148 on B200); 148 when no device is visible,
// so that workspace sizing also answers on a host without a GPU.
int sm_count() {
  static int cached[kMaxDevices] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

// Dynamic shared memory opt-in, once per (kernel, device).
template <typename Kernel>
bool set_smem_once(Kernel kernel, int bytes, bool *done_table) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return false;
  if (!done_table[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return false;
    done_table[dev] = true;
  }
  return true;
}

// Launch with programmatic stream serialization: the kernel may be scheduled
// while the previous kernel in the stream is still running (it calls
// pdl_wait() before touching that kernel's results, common.cuh).  Inside a
// captured CUDA graph the same edge becomes a programmatic dependency.
template <typename... KArgs, typename... Args>
int launch_pdl(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  return e == cudaSuccess ? RIB_OK : rib::host_fail_cuda(what, e);
}

// Makes the stream's device current for this library's runtime, so a launch
// lands on the caller's device whatever this thread's runtime state says.
bool bind_stream_device(void *stream) {
  if (!stream) return true;
  // A stream under graph capture refuses cudaStreamGetDevice (and the refusal
  // invalidates the capture); the capturing caller has its device current.
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cs) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (cs != cudaStreamCaptureStatusNone) return true;
  int dev = -1;
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) {
    cudaGetLastError();
    if (cudaSetDevice(dev) != cudaSuccess) return false;
  }
  return true;
}

// ------------------------------------------------------------------ rope
int rope_launch(const void *qkv, int L, const void *qw, const void *kw, int offset, int nq, int nkv,
                double base, int Lp, void *q_out, void *kv, int kv_rows, int kv_row0, void *stream,
                const int32_t *offset_dev = nullptr, bool rows_follow_offset = true) {
  if (L < 1 || Lp < L || nq < 1 || nkv < 1 || nq + 2 * nkv > rib::rope::kMaxItems || offset < 0 ||
      !(base > 0.0) || kv_rows < 1)
    return RIB_EINVAL;
  if (!qkv || !qw || !kw || !q_out || !kv) return RIB_EINVAL;
  if (!aligned16(qkv) || !aligned16(qw) || !aligned16(kw) || !aligned16(q_out) || !aligned16(kv))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  rib::rope::Params p;
  p.qkv = static_cast<const uint16_t *>(qkv);
  p.qw = static_cast<const uint16_t *>(qw);
  p.kw = static_cast<const uint16_t *>(kw);
  p.q_out = static_cast<uint16_t *>(q_out);
  p.kv = static_cast<uint16_t *>(kv);
  p.L = L;
  p.Lp = Lp;
  p.offset = offset;
  p.nq = nq;
  p.nkv = nkv;
  p.kv_rows = kv_rows;
  p.kv_row0 = kv_row0;
  p.offset_dev = offset_dev;
  p.rows_follow_offset = rows_follow_offset ? 1 : 0;
  rib::rope::rope_inv_freq(p.inv_freq, base);
  const int items = nq + 2 * nkv;
  const int threads = ((items + 1) / 2) * 32;
  // One CTA per token: measured faster on B200 for a 4096-token prompt
  // (20.6 us per layer) than a grid of one wave whose CTAs loop over tokens
  // with the next token's load prefetched (23.5 us).
  return launch_pdl("qk_norm_rope_kernel launch", rib::rope::qk_norm_rope_kernel, dim3(Lp), dim3(threads), 0,
                    static_cast<cudaStream_t>(stream), p);
}

// ------------------------------------------------------------------ decode
struct DecodeGeometry {
  bool streamk;   // stream-K kernel: max_splits = segments per unit, grid = one wave
  int chunk;
  int max_splits;
  int max_groups = 0;  // first-level merge groups per unit (split kernel)
  size_t counters_bytes, ml_bytes, o_bytes, total;
  bool clear_counters;  // counters outside the fixed region: cleared before the launch
};

// Split counters live in a fixed region at the start of every workspace, so a
// workspace shared by calls of different shapes never holds one call's
// partials where another keeps counters.  The kernel leaves every counter it
// used at zero, so once the region is zero (a zero-filled allocation, or
// rib_decode_workspace_init) no call needs a memset before its launch.
constexpr size_t kCounterRegionBytes = 16384;
constexpr size_t kCounterRegionUnits = kCounterRegionBytes / sizeof(int) - 1;

DecodeGeometry split_geometry(int batch, int max_n, int nkv);

// Whether a decode launch runs the stream-K kernel.  Measured on B200
// (28-layer batches, 1-8 KV heads, 1-32k keys, ragged batches of 64 and 200
// sequences): stream-K is faster when the split kernel would run more than
// one wave of short splits (under 96 tiles), as for one-head shards at 32k
// (+8 %), 4k contexts (+22 %) and ragged batches of 512-4096 keys (+6 %);
// the split kernel is faster when its grid is a single wave (one long
// sequence), when its splits are long (2-8 heads at 32k), and when units are
// short (at most 1024 keys: segments cost more than they stream), and when
// the launch holds too few tiles for every CTA of the wave to take
// kStreamMinTiles (a single short sequence).
bool use_streamk(int batch, int max_n, int nkv) {
  using namespace rib::decode;
  const int wave = RIB_DECODE_SLOTS_PER_SM * sm_count();
  if (!RIB_DECODE_STREAMK || batch > kStreamMaxSeqs || wave + 1 > kStreamMaxSegs) return false;
  if (RIB_DECODE_STREAMK == 2) return true;  // build-time override: every launch that fits
  if (max_n <= 1024) return false;
  // enough tiles for every CTA of the wave to take its minimum
  const long long units = static_cast<long long>(batch) * nkv;
  if (units * ceil_div(max_n, TK) < static_cast<long long>(wave) * kStreamMinTiles) return false;
  const DecodeGeometry sg = split_geometry(batch, max_n, nkv);
  return sg.chunk < 96 * TK && units * sg.max_splits > wave;
}

DecodeGeometry decode_geometry(int batch, int max_n, int nkv, bool streamk) {
  using namespace rib::decode;
  if (!streamk) return split_geometry(batch, max_n, nkv);
  DecodeGeometry g;
  g.streamk = true;
  // A unit spans at most one CTA per kStreamMinTiles tiles plus one, and
  // never more CTAs than one wave holds (plus one).
  g.chunk = 0;
  g.max_splits = std::min(stream_max_segments(max_n), RIB_DECODE_SLOTS_PER_SM * sm_count() + 1);
  const size_t units = static_cast<size_t>(batch) * nkv;
  g.clear_counters = units > kCounterRegionUnits;
  g.counters_bytes = g.clear_counters ? (((units + 1) * sizeof(int) + 255) / 256) * 256 : kCounterRegionBytes;
  g.ml_bytes = ((units * g.max_splits * 2 * 2 * sizeof(float) + 255) / 256) * 256;
  g.o_bytes = units * g.max_splits * 2 * D * sizeof(float);
  g.total = g.counters_bytes + g.ml_bytes + g.o_bytes;
  return g;
}

DecodeGeometry split_geometry(int batch, int max_n, int nkv) {
  using namespace rib::decode;
  DecodeGeometry g;
  g.streamk = false;
  // Split count: start from the larger of "chunks of at most
  // RIB_DECODE_MAX_CHUNK keys" and
  // "at least one full wave of 2 CTAs per SM", then take the smallest count
  // up to twice that whose CTA total fills whole waves (>= 97% of the last
  // wave's slots), so no nearly empty wave trails the launch; otherwise the
  // best wave fill in that range.
  const long long slots = static_cast<long long>(RIB_DECODE_SLOTS_PER_SM) * sm_count();
  const long long n_units = static_cast<long long>(batch) * nkv;
  const int lo = std::max(ceil_div(max_n, RIB_DECODE_MAX_CHUNK),
                          std::min(ceil_div(RIB_DECODE_MIN_WAVES * slots, n_units), ceil_div(max_n, TK)));
  const int hi = std::max(lo, std::min(2 * lo, ceil_div(max_n, TK)));
  int best_chunk = ceil_div(ceil_div(max_n, lo), TK) * TK;
  double best_eff = -1.0;
  for (int splits = lo; splits <= hi; ++splits) {
    const int chunk = max(TK, ceil_div(ceil_div(max_n, splits), TK) * TK);
    const long long ctas = n_units * ceil_div(max_n, chunk);
    const long long waves = (ctas + slots - 1) / slots;
    const double eff = static_cast<double>(ctas) / static_cast<double>(waves * slots);
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best_chunk = chunk;
    }
    if (eff >= 0.97) break;
  }
  g.chunk = best_chunk;
  g.max_splits = ceil_div(max_n, best_chunk);
  g.max_groups = ceil_div(g.max_splits, kMergeGroup);
  const size_t units = static_cast<size_t>(batch) * nkv;
  // per-unit split counters, one counter of units finalised (all-gather),
  // then per-unit counters of the first-level merge groups
  const size_t n_counters = units + 1 + units * g.max_groups;
  g.clear_counters = n_counters * sizeof(int) > kCounterRegionBytes;
  g.counters_bytes = g.clear_counters ? ((n_counters * sizeof(int) + 255) / 256) * 256 : kCounterRegionBytes;
  g.ml_bytes = ((units * g.max_splits * 2 * 2 * sizeof(float) + 255) / 256) * 256;
  g.o_bytes = units * g.max_splits * 2 * D * sizeof(float);
  g.total = g.counters_bytes + g.ml_bytes + g.o_bytes;
  return g;
}

bool g_decode_smem_done[kMaxDevices];
bool g_streamk_smem_done[kMaxDevices];

// allow_streamk: false for callers whose scratch is sized for the split
// kernel (the no-allocation entry point).
int decode_launch(rib::decode::Params p, int batch, int max_n, void *workspace, size_t workspace_bytes,
                  void *stream, bool allow_streamk = true) {
  using namespace rib::decode;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const DecodeGeometry g = decode_geometry(batch, max_n, p.nkv, allow_streamk && use_streamk(batch, max_n, p.nkv));
  if (!workspace || workspace_bytes < g.total) return RIB_EINVAL;
  if (!aligned16(workspace)) return RIB_EALIGN;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  // The split counters must start at zero.  In the fixed region they do (the
  // workspace contract; the kernel resets what it uses); a launch with more
  // units than the region holds clears its own, larger region first.
  if (g.clear_counters) {
    const cudaError_t ze = cudaMemsetAsync(ws, 0, g.counters_bytes, static_cast<cudaStream_t>(stream));
    if (ze != cudaSuccess) return rib::host_fail_cuda("cudaMemsetAsync(decode counters)", ze);
  }
  p.counters = reinterpret_cast<int *>(ws);
  p.done = p.counters + static_cast<size_t>(batch) * p.nkv;
  p.gcounters = p.done + 1;
  p.max_groups = g.max_groups;
  if (!g.streamk && g.max_groups > kMergeSplits) return RIB_EINVAL;  // beyond any cache that fits a GPU
  p.part_ml = reinterpret_cast<float *>(ws + g.counters_bytes);
  p.part_o = reinterpret_cast<float *>(ws + g.counters_bytes + g.ml_bytes);
  p.chunk = g.chunk;
  p.max_splits = g.max_splits;
  p.max_n = max_n;
  if (g.streamk) {
    const int smem = static_cast<int>(sizeof(StreamSmem)) + 128;
    if (!set_smem_once(decode_streamk_kernel, smem, g_streamk_smem_done))
      return rib::host_fail(RIB_ECUDA, "cudaFuncSetAttribute(decode stream-K smem)", 0);
    return launch_pdl("decode_streamk_kernel launch", decode_streamk_kernel,
                      dim3(RIB_DECODE_SLOTS_PER_SM * sm_count()), dim3(NTHREADS), smem,
                      static_cast<cudaStream_t>(stream), p, batch);
  }
  const int smem = static_cast<int>(sizeof(Smem)) + 128;
  if (!set_smem_once(decode_kernel, smem, g_decode_smem_done))
    return rib::host_fail(RIB_ECUDA, "cudaFuncSetAttribute(decode smem)", 0);
  dim3 grid(g.max_splits, p.nkv, batch);
  return launch_pdl("decode_kernel launch", decode_kernel, grid, dim3(NTHREADS), smem,
                    static_cast<cudaStream_t>(stream), p);
}

// ------------------------------------------------------------------ decode, no allocation
// Scratch of rib_decode_attention_noalloc: a fixed array in the library's own
// device memory, so that entry point needs no workspace from the caller.
// Every GPU that loads the library holds it until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // 2 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void *g_noalloc_scratch_addr[kMaxDevices];  // device address of the array, per device

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device with cudaGetSymbolAddress.
void *noalloc_scratch(int dev) {
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_scratch_addr[dev]) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
      rib::host_fail_cuda("cudaGetSymbolAddress(g_noalloc_scratch)", e);
      return nullptr;
    }
    g_noalloc_scratch_addr[dev] = ptr;
  }
  return g_noalloc_scratch_addr[dev];
}

// ------------------------------------------------------------------ model kernels
template <int R, int C, bool SW, bool TP>
int gemv_launch_rc(const rib::model::GemvParams &p, cudaStream_t st, bool wide) {
  using rib::model::kGemvWarps;
  using rib::model::kGemvWideWarps;
  if constexpr (R == 1 && C > 0 && !TP) {
    if (wide) {
      const int grid = ceil_div(p.rows_out, kGemvWideWarps * R);
      return launch_pdl("gemv_kernel launch", rib::model::gemv_kernel<R, C, SW, TP, kGemvWideWarps>,
                        dim3(grid), dim3(kGemvWideWarps * 32), p.K * sizeof(float), st, p);
    }
  }
  const int grid = ceil_div(p.rows_out, kGemvWarps * R);
  return launch_pdl("gemv_kernel launch", rib::model::gemv_kernel<R, C, SW, TP>, dim3(grid),
                    dim3(kGemvWarps * 32), p.K * sizeof(float), st, p);
}

// Compile-time chunk counts for the K of Qwen3 projections, whole and split
// over 2, 4 or 8 ranks; other K take the runtime loop.
template <int R, bool SW, bool TP>
int gemv_launch_r(const rib::model::GemvParams &p, cudaStream_t st, bool wide) {
  switch (p.K) {
    case 256: return gemv_launch_rc<R, 1, SW, TP>(p, st, wide);
    case 512: return gemv_launch_rc<R, 2, SW, TP>(p, st, wide);
    case 768: return gemv_launch_rc<R, 3, SW, TP>(p, st, wide);
    case 1024: return gemv_launch_rc<R, 4, SW, TP>(p, st, wide);
    case 1536: return gemv_launch_rc<R, 6, SW, TP>(p, st, wide);
    case 2048: return gemv_launch_rc<R, 8, SW, TP>(p, st, wide);
    case 3072: return gemv_launch_rc<R, 12, SW, TP>(p, st, wide);
    default: return gemv_launch_rc<R, 0, SW, TP>(p, st, wide);
  }
}

template <int R>
int gemv_launch_r(const rib::model::GemvParams &p, cudaStream_t st, bool wide) {
  const bool tp = p.in_sum || p.epi == rib::model::kPeerPartial;
  if (p.epi == rib::model::kSwiGLU)
    return tp ? gemv_launch_r<R, true, true>(p, st, wide) : gemv_launch_r<R, true, false>(p, st, wide);
  return tp ? gemv_launch_r<R, false, true>(p, st, wide) : gemv_launch_r<R, false, false>(p, st, wide);
}

// ------------------------------------------------------------------ persistent decode step
inline size_t round256(size_t b) { return (b + 255) / 256 * 256; }

struct StepLayout {
  DecodeGeometry g;
  size_t sync_off, ml_off, po_off, h_off[3], qkv_off, q_off, ao_off, a_off, total;
};

StepLayout step_layout(const rib_qwen3_model *m, int cap) {
  StepLayout l;
  l.g = split_geometry(1, cap, m->num_kv_heads);
  size_t off = kCounterRegionBytes;  // decode split counters (fixed region)
  l.sync_off = off;
  off += round256(sizeof(rib::step::Sync));
  l.ml_off = off;
  off += round256(l.g.ml_bytes);
  l.po_off = off;
  off += round256(l.g.o_bytes);
  for (int i = 0; i < 3; ++i) {
    l.h_off[i] = off;
    off += round256(static_cast<size_t>(m->hidden) * 2);
  }
  l.qkv_off = off;
  off += round256(static_cast<size_t>(m->num_heads + 2 * m->num_kv_heads) * 128 * 2);
  l.q_off = off;
  off += round256(static_cast<size_t>(m->num_heads) * 128 * 2);
  l.ao_off = off;
  off += round256(static_cast<size_t>(m->num_heads) * 128 * 2);
  l.a_off = off;
  off += round256(static_cast<size_t>(m->intermediate) * 2);
  l.total = off;
  return l;
}

bool step_model_ok(const rib_qwen3_model *m) {
  if (!m || m->num_layers < 1 || m->num_layers > RIB_QWEN3_MAX_LAYERS || m->num_kv_heads < 1 ||
      m->num_heads != 2 * m->num_kv_heads || m->num_heads + 2 * m->num_kv_heads > rib::rope::kMaxItems ||
      m->hidden < 256 || m->hidden % 256 || m->hidden > rib::model::kMaxK || m->intermediate < 256 ||
      m->intermediate % 256 || m->intermediate > rib::model::kMaxK || (m->num_heads * 128) % 256 ||
      m->num_heads * 128 > rib::model::kMaxK || m->vocab < 1 || !(m->rope_theta > 0.0))
    return false;
  return m->embed && m->final_norm;
}

bool g_step_smem_done[2][kMaxDevices];

template <int CH, int CQ, int CI, int MQ, int MO, int MG, int MD>
int step_launch(const rib::step::Params &p, int which, cudaStream_t st) {
  auto kernel = rib::step::decode_step_kernel<CH, CQ, CI, MQ, MO, MG, MD>;
  const int smem = static_cast<int>(sizeof(rib::decode::Smem)) + 128;
  if (!set_smem_once(kernel, smem, g_step_smem_done[which]))
    return rib::host_fail(RIB_ECUDA, "cudaFuncSetAttribute(decode step smem)", 0);
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, rib::step::NT, smem);
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaOccupancyMaxActiveBlocksPerMultiprocessor(decode step)", e);
  if (per_sm < 1) return rib::host_fail(RIB_ECUDA, "decode step kernel does not fit on an SM", per_sm);
  per_sm = std::min(per_sm, RIB_DECODE_SLOTS_PER_SM);
  if (per_sm * sm_count() > rib::step::kMaxCtas)
    return rib::host_fail(RIB_ECUDA, "decode step grid exceeds the barrier slots", per_sm * sm_count());
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(per_sm * sm_count());
  cfg.blockDim = dim3(rib::step::NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barrier relies on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kernel, p);
  return e == cudaSuccess ? RIB_OK : rib::host_fail_cuda("decode_step_kernel launch", e);
}

// ------------------------------------------------------------------ GEMM (prefill projections)
// 2-D BF16 map of a row-major [rows][cols] matrix (row stride ld elements),
// box (64 columns, box_rows rows), 128-byte swizzle; rows past `rows` read
// as zero.
bool gemm_map(CUtensorMap *m, const void *base, long long rows, long long cols, long long ld, int box_rows) {
  rib::prefill::EncodeTiledFn enc = rib::prefill::encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    rib::host_fail(RIB_ECUDA, "cuTensorMapEncodeTiled (gemm)", static_cast<int>(r));
    return false;
  }
  return true;
}

bool g_gemm_smem_done[3][kMaxDevices];

template <int BN, int MH>
int gemm_launch_bn(rib::gemm::Params &p, const void *A, const void *W, int w_box_rows, cudaStream_t st) {
  using namespace rib::gemm;
  if (!gemm_map(&p.tm_a, A, p.M, p.K, p.K, BM * MH) || !gemm_map(&p.tm_b, W, p.N, p.K, p.K, w_box_rows))
    return RIB_ECUDA;
  const int smem = static_cast<int>(sizeof(Smem<BN, MH>)) + 1024;
  if (!set_smem_once(gemm_kernel<BN, MH>, smem, g_gemm_smem_done[MH == 2 ? 2 : BN == 256]))
    return rib::host_fail(RIB_ECUDA, "cudaFuncSetAttribute(gemm smem)", smem);
  const int grid = std::min(p.num_tiles, sm_count());
  return launch_pdl("gemm_kernel launch", gemm_kernel<BN, MH>, dim3(grid), dim3(NTHREADS), smem, st, p);
}

// Shared checks and launch of every GEMM entry point.  256-row tiles (two
// accumulator halves sharing each W stage) for the plain BF16 / FP32 stores
// when N takes 256-wide tiles and there are at least as many such tiles as
// SMs; else 128-row tiles, whose two accumulators let the epilogue of one
// tile run under the next tile's MMAs (the SwiGLU and QK-norm + RoPE
// epilogues take about as long as a tile's MMAs).
int gemm_run(const void *A, int M, int K, const void *W, int N, int epi, int bn, rib::gemm::Params &p,
             void *stream) {
  using namespace rib::gemm;
  if (!A || !W || M < 1 || N < 1 || K < BK || K % BK) return RIB_EINVAL;
  if (epi == kSwiGLU || epi == kQKRope ? N % bn : N % 8) return RIB_EINVAL;
  if (!aligned16(A) || !aligned16(W)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  p.M = M;
  p.N = N;
  p.K = K;
  p.epi = epi;
  const int out_cols = epi == kSwiGLU ? N / 2 : N;
  const int ntiles_n = epi == kSwiGLU ? out_cols / 128 : ceil_div(N, bn);
  const bool two_halves = bn == 256 && (epi == kBF16 || epi == kF32) && ceil_div(M, 2 * BM) * ntiles_n >= sm_count();
  p.num_m = ceil_div(M, two_halves ? 2 * BM : BM);
  p.num_tiles = p.num_m * ntiles_n;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int w_rows = epi == kSwiGLU ? 128 : bn;
  if (two_halves) return gemm_launch_bn<256, 2>(p, A, W, w_rows, st);
  if (bn == 256) return gemm_launch_bn<256, 1>(p, A, W, w_rows, st);
  return gemm_launch_bn<128, 1>(p, A, W, w_rows, st);
}

}  // namespace

extern "C" {

int rib_version(void) { return (1 << 16) | 0; }

const char *rib_status_string(int status) {
  switch (status) {
    case RIB_OK: return "ok";
    case RIB_EINVAL: return "invalid argument or shape";
    case RIB_ECAPACITY: return "KV capacity exceeded";
    case RIB_EALIGN: return "pointer not 16-byte aligned";
    case RIB_ECUDA: return "CUDA runtime error";
    case RIB_ETIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

const char *rib_last_error_string(void) { return rib::g_last_error; }

int rib_take_device_status(int *status_host) {
  if (!status_host) return RIB_EINVAL;
  if (cudaDeviceSynchronize() != cudaSuccess) return RIB_ECUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, rib::g_device_status, sizeof(int)) != cudaSuccess) return RIB_ECUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(rib::g_device_status, &zero, sizeof(int)) != cudaSuccess) return RIB_ECUDA;
  *status_host = v;
  return RIB_OK;
}

int rib_set_wait_limit_ns(unsigned long long ns) {
  if (ns < 1000000ull || ns > 60000000000ull) return RIB_EINVAL;
  const cudaError_t e = cudaMemcpyToSymbol(rib::g_wait_limit_ns, &ns, sizeof(ns));
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaMemcpyToSymbol(wait limit)", e);
  return RIB_OK;
}

int rib_get_wait_limit_ns(unsigned long long *ns) {
  if (!ns) return RIB_EINVAL;
  const cudaError_t e = cudaMemcpyFromSymbol(ns, rib::g_wait_limit_ns, sizeof(*ns));
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaMemcpyFromSymbol(wait limit)", e);
  return RIB_OK;
}

int rib_qk_norm_rope(const void *qkv, const void *qw, const void *kw, int pos, int nq, int nkv,
                     double base, void *q_out, void *kv_out, void *stream) {
  return rope_launch(qkv, 1, qw, kw, pos, nq, nkv, base, 1, q_out, kv_out, 1, 0, stream);
}

int rib_qk_norm_rope_prefill(const void *qkv, int L, const void *qw, const void *kw, int offset,
                             int nq, int nkv, double base, int Lp, void *q_out, void *kv_out,
                             void *stream) {
  return rope_launch(qkv, L, qw, kw, offset, nq, nkv, base, Lp, q_out, kv_out, L, 0, stream);
}

int rib_qk_norm_rope_append(const void *qkv, int L, const void *qw, const void *kw, int offset,
                            int nq, int nkv, double base, int Lp, void *q_out, void *cache,
                            int cap, void *stream) {
  if (L < 1 || offset < 0 || cap < 1) return RIB_EINVAL;
  if (static_cast<long long>(offset) + L > cap) return RIB_ECAPACITY;
  return rope_launch(qkv, L, qw, kw, offset, nq, nkv, base, Lp, q_out, cache, cap, offset, stream);
}

size_t rib_decode_workspace_bytes(int batch, int max_n, int nkv) {
  if (batch < 1 || max_n < 1 || nkv < 1) return 0;
  // the larger of the two kernels' needs: entry points that force the split
  // kernel (rib_decode_attention_qkv) take the same workspace
  return std::max(split_geometry(batch, max_n, nkv).total,
                  decode_geometry(batch, max_n, nkv, use_streamk(batch, max_n, nkv)).total);
}

int rib_decode_kernel_choice(int batch, int max_n, int nkv) {
  if (batch < 1 || max_n < 1 || nkv < 1) return -RIB_EINVAL;
  return use_streamk(batch, max_n, nkv) ? 1 : 0;
}

int rib_decode_workspace_init(void *workspace, size_t workspace_bytes, void *stream) {
  if (!workspace || workspace_bytes < kCounterRegionBytes) return RIB_EINVAL;
  if (!aligned16(workspace)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const cudaError_t e = cudaMemsetAsync(workspace, 0, kCounterRegionBytes, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? RIB_OK : rib::host_fail_cuda("cudaMemsetAsync(decode workspace init)", e);
}

int rib_decode_attention(const void *q, const void *cache, int cap, int n, int nq, int nkv,
                         float scale, void *out, void *workspace, size_t workspace_bytes,
                         void *stream) {
  if (!q || !cache || !out) return RIB_EINVAL;
  if (nkv < 1 || nq != 2 * nkv || n < 1 || cap < 1 || !(scale > 0.f)) return RIB_EINVAL;
  if (n > cap) return RIB_ECAPACITY;
  if (!aligned16(q) || !aligned16(cache) || !aligned16(out)) return RIB_EALIGN;
  rib::decode::Params p = {};
  p.q = static_cast<const uint16_t *>(q);
  p.cache = static_cast<const uint16_t *>(cache);
  p.cache_ptrs = nullptr;
  p.lens = nullptr;
  p.n_single = n;
  p.cap = cap;
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t *>(out);
  return decode_launch(p, 1, n, workspace, workspace_bytes, stream);
}

int rib_decode_attention_noalloc(const void *q, const void *cache, int cap, int n, int nq, int nkv,
                                 float scale, void *out, void *stream) {
  if (!q || !cache || !out) return RIB_EINVAL;
  if (nkv < 1 || nq != 2 * nkv || n < 1 || cap < 1 || !(scale > 0.f)) return RIB_EINVAL;
  if (n > cap) return RIB_ECAPACITY;
  if (!aligned16(q) || !aligned16(cache) || !aligned16(out)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const DecodeGeometry g = split_geometry(1, n, nkv);
  if (g.total > kNoAllocScratchBytes) {
    snprintf(rib::g_last_error, sizeof(rib::g_last_error),
             "rib_decode_attention_noalloc: n=%d with %d KV heads needs %zu bytes of scratch, "
             "more than the %zu-byte static scratch", n, nkv, g.total, kNoAllocScratchBytes);
    return RIB_EINVAL;
  }
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return rib::host_fail(RIB_ECUDA, "cudaGetDevice", dev);
  void *scratch = noalloc_scratch(dev);
  if (!scratch) return RIB_ECUDA;
  // (decode_launch clears the split counters on the stream before launching.)
  rib::decode::Params p = {};
  p.q = static_cast<const uint16_t *>(q);
  p.cache = static_cast<const uint16_t *>(cache);
  p.cache_ptrs = nullptr;
  p.lens = nullptr;
  p.n_single = n;
  p.cap = cap;
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t *>(out);
  return decode_launch(p, 1, n, scratch, kNoAllocScratchBytes, stream, false);
}

size_t rib_peer_buffer_bytes(int batch, int nq_total) {
  if (batch < 1 || nq_total < 1) return 0;
  const size_t region = ((static_cast<size_t>(batch) * nq_total * 128 * 2 + 255) / 256) * 256;
  return 2 * region + 256;  // two output regions, then the signal slots
}

int rib_peer_buffer_alloc(int device, size_t bytes, void **dev_ptr, void *ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return RIB_EINVAL;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaSetDevice", e);
  void *ptr = nullptr;
  if ((e = cudaMalloc(&ptr, bytes)) != cudaSuccess) return rib::host_fail_cuda("cudaMalloc(peer buffer)", e);
  if ((e = cudaMemset(ptr, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
    cudaFree(ptr);
    return rib::host_fail_cuda("cudaMemset(peer buffer)", e);
  }
  if ((e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), ptr)) != cudaSuccess) {
    cudaFree(ptr);
    return rib::host_fail_cuda("cudaIpcGetMemHandle", e);
  }
  *dev_ptr = ptr;
  return RIB_OK;
}

int rib_peer_buffer_open(int device, const void *ipc_handle, void **peer_ptr) {
  if (!ipc_handle || !peer_ptr) return RIB_EINVAL;
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaSetDevice", e);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  if ((e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess)
    return rib::host_fail_cuda("cudaIpcOpenMemHandle", e);
  return RIB_OK;
}

int rib_peer_buffer_close(int device, void *peer_ptr) {
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? RIB_OK : rib::host_fail_cuda("cudaIpcCloseMemHandle", e);
}

int rib_peer_buffer_free(int device, void *dev_ptr) {
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaFree(dev_ptr);
  return e == cudaSuccess ? RIB_OK : rib::host_fail_cuda("cudaFree(peer buffer)", e);
}

int rib_decode_attention_gather(const void *q, const uint64_t *cache_ptrs, const int32_t *lens,
                                int batch, int max_n, int cap, int nq, int nkv, float scale,
                                const rib_peer_gather *g, unsigned long long epoch,
                                void *workspace, size_t workspace_bytes, void *stream) {
  if (!q || !cache_ptrs || !lens || !g) return RIB_EINVAL;
  if (batch < 1 || nkv < 1 || nq != 2 * nkv || max_n < 1 || cap < 1 || !(scale > 0.f))
    return RIB_EINVAL;
  if (g->world < 1 || g->world > RIB_MAX_PEERS || g->rank < 0 || g->rank >= g->world || epoch == 0)
    return RIB_EINVAL;
  if (g->region_bytes < static_cast<size_t>(batch) * g->world * nq * 128 * 2) return RIB_EINVAL;
  if (max_n > cap) return RIB_ECAPACITY;
  if (!aligned16(q) || (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u) ||
      (reinterpret_cast<uintptr_t>(lens) & 3u))
    return RIB_EALIGN;
  rib::decode::Params p = {};
  for (int r = 0; r < g->world; ++r) {
    if (!g->out[r] || !g->sig[r] || (g->out[r] & 15u) || (g->sig[r] & 7u)) return RIB_EALIGN;
    p.gout[r] = reinterpret_cast<uint16_t *>(g->out[r] + (epoch & 1ull) * g->region_bytes);
    p.gsig[r] = reinterpret_cast<unsigned long long *>(g->sig[r]);
  }
  p.q = static_cast<const uint16_t *>(q);
  p.cache = nullptr;
  p.cache_ptrs = cache_ptrs;
  p.lens = lens;
  p.cap = cap;
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = nullptr;
  p.world = g->world;
  p.rank = g->rank;
  p.nq_total = g->world * nq;
  p.epoch = epoch;
  p.total_units = batch * nkv;
  // Early ring fill (header: lens, cache_ptrs and the cache rows below the
  // new token's are complete at launch): a call's first tiles stream while
  // the previous call finishes its exchange with the peers.
  p.early = 1;
  return decode_launch(p, batch, max_n, workspace, workspace_bytes, stream);
}

int rib_decode_attention_gather_dev(const void *q, const uint64_t *cache_ptrs, const int32_t *lens,
                                    int batch, int max_n, int cap, int nq, int nkv, float scale,
                                    const rib_peer_gather *g, unsigned long long *epoch_dev,
                                    void *out_copy, void *workspace, size_t workspace_bytes, void *stream) {
  if (!q || !cache_ptrs || !lens || !g || !epoch_dev || !out_copy) return RIB_EINVAL;
  if (batch < 1 || nkv < 1 || nq != 2 * nkv || max_n < 1 || cap < 1 || !(scale > 0.f))
    return RIB_EINVAL;
  if (g->world < 1 || g->world > RIB_MAX_PEERS || g->rank < 0 || g->rank >= g->world) return RIB_EINVAL;
  const size_t elems = static_cast<size_t>(batch) * g->world * nq * 128;
  if (g->region_bytes < elems * 2 || (g->region_bytes & 15u)) return RIB_EINVAL;
  if (max_n > cap) return RIB_ECAPACITY;
  if (!aligned16(q) || !aligned16(out_copy) || (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u) ||
      (reinterpret_cast<uintptr_t>(lens) & 3u) || (reinterpret_cast<uintptr_t>(epoch_dev) & 7u))
    return RIB_EALIGN;
  rib::decode::Params p = {};
  for (int r = 0; r < g->world; ++r) {
    if (!g->out[r] || !g->sig[r] || (g->out[r] & 15u) || (g->sig[r] & 7u)) return RIB_EALIGN;
    p.gout[r] = reinterpret_cast<uint16_t *>(g->out[r]);
    p.gsig[r] = reinterpret_cast<unsigned long long *>(g->sig[r]);
  }
  p.q = static_cast<const uint16_t *>(q);
  p.cache = nullptr;
  p.cache_ptrs = cache_ptrs;
  p.lens = lens;
  p.cap = cap;
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = nullptr;
  p.world = g->world;
  p.rank = g->rank;
  p.nq_total = g->world * nq;
  p.epoch = 0;
  p.epoch_dev = epoch_dev;
  p.region_elems = g->region_bytes / 2;
  p.gcopy = static_cast<uint16_t *>(out_copy);
  p.total_units = batch * nkv;
  return decode_launch(p, batch, max_n, workspace, workspace_bytes, stream);
}

int rib_decode_attention_batched(const void *q, const uint64_t *cache_ptrs, const int32_t *lens,
                                 int batch, int max_n, int cap, int nq, int nkv, float scale,
                                 void *out, void *workspace, size_t workspace_bytes, void *stream) {
  if (!q || !cache_ptrs || !lens || !out) return RIB_EINVAL;
  if (batch < 1 || nkv < 1 || nq != 2 * nkv || max_n < 1 || cap < 1 || !(scale > 0.f))
    return RIB_EINVAL;
  if (max_n > cap) return RIB_ECAPACITY;
  if (!aligned16(q) || !aligned16(out) || (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u) ||
      (reinterpret_cast<uintptr_t>(lens) & 3u))
    return RIB_EALIGN;
  rib::decode::Params p = {};
  p.q = static_cast<const uint16_t *>(q);
  p.cache = nullptr;
  p.cache_ptrs = cache_ptrs;
  p.lens = lens;
  p.n_single = 0;
  p.cap = cap;
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t *>(out);
  return decode_launch(p, batch, max_n, workspace, workspace_bytes, stream);
}

int rib_decode_attention_qkv(const void *qkv, const void *qw, const void *kw, double base,
                             const uint64_t *cache_ptrs, const int32_t *lens, int batch, int max_n, int cap,
                             int nq, int nkv, float scale, void *out, void *workspace, size_t workspace_bytes,
                             void *stream) {
  if (!qkv || !qw || !kw || !cache_ptrs || !lens || !out) return RIB_EINVAL;
  if (batch < 1 || nkv < 1 || nq != 2 * nkv || nq + 2 * nkv > rib::rope::kMaxItems || max_n < 1 || cap < 1 ||
      !(scale > 0.f) || !(base > 0.0))
    return RIB_EINVAL;
  if (max_n > cap) return RIB_ECAPACITY;
  if (!aligned16(qkv) || !aligned16(qw) || !aligned16(kw) || !aligned16(out) ||
      (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u) || (reinterpret_cast<uintptr_t>(lens) & 3u))
    return RIB_EALIGN;
  rib::decode::Params p = {};
  p.q = static_cast<const uint16_t *>(qkv);  // (q is formed from qkv in the kernel)
  p.qkv = static_cast<const uint16_t *>(qkv);
  p.early = 1;
  p.qw = static_cast<const uint16_t *>(qw);
  p.kw = static_cast<const uint16_t *>(kw);
  rib::rope::rope_inv_freq(p.inv_freq, base);
  p.cache = nullptr;
  p.cache_ptrs = cache_ptrs;
  p.lens = lens;
  p.cap = cap;
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t *>(out);
  return decode_launch(p, batch, max_n, workspace, workspace_bytes, stream, false);
}

size_t rib_prefill_workspace_bytes(int kL, int nkv) {
  if (kL < 1 || nkv < 1) return 0;
  return rib::prefill::workspace_bytes(kL, nkv);
}

int rib_prefill_attention(const void *Q, const void *K, const void *V, int qL, int kL, int qLp,
                          int cap, int H, int nkv, float scale, void *O, void *workspace,
                          size_t workspace_bytes, void *stream) {
  return rib::prefill::launch(Q, K, V, qL, kL, qLp, cap, H, nkv, scale, O, workspace, workspace_bytes,
                              stream, bind_stream_device);
}


// ------------------------------------------------------------------ model kernels
int rib_qk_norm_rope_prefill_dev(const void *qkv, int L, const void *qw, const void *kw,
                                 const int32_t *offset_dev, int nq, int nkv, double base, int Lp,
                                 void *q_out, void *kv_out, void *stream) {
  if (L < 1 || !offset_dev) return RIB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(offset_dev) & 3u)) return RIB_EALIGN;
  return rope_launch(qkv, L, qw, kw, 0, nq, nkv, base, Lp, q_out, kv_out, L, 0, stream, offset_dev, false);
}

int rib_qk_norm_rope_append_dev(const void *qkv, int L, const void *qw, const void *kw,
                                const int32_t *offset_dev, int nq, int nkv, double base, int Lp,
                                void *q_out, void *cache, int cap, void *stream) {
  if (L < 1 || cap < 1 || !offset_dev) return RIB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(offset_dev) & 3u)) return RIB_EALIGN;
  return rope_launch(qkv, L, qw, kw, 0, nq, nkv, base, Lp, q_out, cache, cap, 0, stream, offset_dev);
}

// Rows per warp: one while that still gives at least 4 CTAs per SM, more for
// tall matrices (the LM head) so that each CTA's x load and norm are
// amortised over more weight bytes.
// wide: the RIB_GEMV_WIDE hint, honoured for one-row-per-warp shapes with a
// compile-time chunk count outside tensor parallelism.
static int gemv_dispatch(const rib::model::GemvParams &p, cudaStream_t st, bool wide = false) {
  using rib::model::kGemvWarps;
  const int target_ctas = 4 * sm_count();
  if (p.rows_out >= target_ctas * kGemvWarps * 4) return gemv_launch_r<4>(p, st, false);
  if (p.rows_out >= target_ctas * kGemvWarps * 2) return gemv_launch_r<2>(p, st, false);
  return gemv_launch_r<1>(p, st, wide);
}

int rib_gemv(const void *W, int N, int K, const void *x, const void *nw, const void *res, int epi,
             int out_f32, void *y, void *stream) {
  using namespace rib::model;
  const bool wide = (epi & RIB_GEMV_WIDE) != 0;
  epi &= ~RIB_GEMV_WIDE;
  if (!W || !x || !y || N < 1 || K < 8 || K % 8 || K > kMaxK) return RIB_EINVAL;
  if (epi != kNone && epi != kResidual && epi != kSwiGLU) return RIB_EINVAL;
  if ((epi == kResidual) != (res != nullptr)) return RIB_EINVAL;
  if (epi == kSwiGLU && (N % 2 || out_f32)) return RIB_EINVAL;
  if (epi == kResidual && out_f32) return RIB_EINVAL;
  if (!aligned16(W) || !aligned16(x) || (nw && !aligned16(nw)) || !aligned16(y) ||
      (res && (reinterpret_cast<uintptr_t>(res) & 1u)))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  GemvParams p = {};
  p.W = static_cast<const uint16_t *>(W);
  p.x = static_cast<const uint16_t *>(x);
  p.nw = static_cast<const uint16_t *>(nw);
  p.res = static_cast<const uint16_t *>(res);
  p.y = y;
  p.N = N;
  p.K = K;
  p.rows_out = epi == kSwiGLU ? N / 2 : N;
  p.epi = epi;
  p.out_f32 = out_f32 ? 1 : 0;
  return gemv_dispatch(p, static_cast<cudaStream_t>(stream), wide);
}

size_t rib_tp_buffer_bytes(int world, int slot) {
  if (world < 1 || world > RIB_TP_MAX_RANKS || slot < 4 || slot % 4) return 0;
  return round256(2 * static_cast<size_t>(world) * slot * sizeof(unsigned long long));
}

// Checks a rib_tp_exchange and converts it to the device form.
static int tp_ex_from(const rib_tp_exchange *ex, rib::model::TpEx &d) {
  if (!ex || ex->world < 1 || ex->world > RIB_TP_MAX_RANKS || ex->rank < 0 || ex->rank >= ex->world ||
      ex->slot < 4 || ex->slot % 4 || !ex->epoch || !ex->done)
    return RIB_EINVAL;
  if ((ex->epoch & 7u) || (ex->done & 3u)) return RIB_EALIGN;
  d = {};
  d.world = ex->world;
  d.rank = ex->rank;
  d.slot = ex->slot;
  for (int q = 0; q < ex->world; ++q) {
    if (!ex->buf[q]) return RIB_EINVAL;
    if (ex->buf[q] & 255u) return RIB_EALIGN;
    d.buf[q] = reinterpret_cast<unsigned long long *>(ex->buf[q]);
  }
  d.epoch = reinterpret_cast<unsigned long long *>(ex->epoch);
  d.done = reinterpret_cast<unsigned int *>(ex->done);
  return RIB_OK;
}

int rib_gemv_tp(const void *W, int N, int K, const void *x, const void *nw, int epi, int out_f32, void *y,
                const rib_tp_exchange *ex, int in_sum, void *x_out, void *stream) {
  using namespace rib::model;
  if (!W || !x || N < 1 || K < 8 || K % 8 || K > kMaxK) return RIB_EINVAL;
  if (epi != kNone && epi != kSwiGLU && epi != kPeerPartial) return RIB_EINVAL;
  if (epi != kPeerPartial && !y) return RIB_EINVAL;
  if (out_f32 && epi != kNone) return RIB_EINVAL;
  if (epi == kSwiGLU && N % 2) return RIB_EINVAL;
  GemvParams p = {};
  if (epi == kPeerPartial || in_sum) {
    const int st = tp_ex_from(ex, p.ex);
    if (st != RIB_OK) return st;
    if ((epi == kPeerPartial && N > ex->slot) || (in_sum && (K > ex->slot || !x_out))) return RIB_EINVAL;
  }
  if (!aligned16(W) || !aligned16(x) || (nw && !aligned16(nw)) || (y && !aligned16(y)) ||
      (in_sum && !aligned16(x_out)))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  p.W = static_cast<const uint16_t *>(W);
  p.x = static_cast<const uint16_t *>(x);
  p.nw = static_cast<const uint16_t *>(nw);
  p.y = y;
  p.N = N;
  p.K = K;
  p.rows_out = epi == kSwiGLU ? N / 2 : N;
  p.epi = epi;
  p.out_f32 = out_f32 ? 1 : 0;
  p.in_sum = in_sum ? 1 : 0;
  p.x_out = static_cast<uint16_t *>(x_out);
  return gemv_dispatch(p, static_cast<cudaStream_t>(stream));
}

int rib_argmax_f32_tp(const float *x, int n, int index_offset, int32_t *out, void *workspace,
                      const rib_tp_exchange *ex, void *stream) {
  if (!x || !out || !workspace || n < 1 || index_offset < 0) return RIB_EINVAL;
  rib::model::TpEx d;
  const int s = tp_ex_from(ex, d);
  if (s != RIB_OK) return s;
  if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15u))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(rib::model::ArgmaxWs), st);
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaMemsetAsync(argmax workspace)", e);
  const int grid = std::max(1, std::min(ceil_div(n, 1024 * 4), sm_count()));
  return launch_pdl("argmax_tp_kernel launch", rib::model::argmax_tp_kernel, dim3(grid), dim3(1024), 0, st, x,
                    n, index_offset, static_cast<rib::model::ArgmaxWs *>(workspace), out, d);
}

// ------------------------------------------------------------------ tensor-parallel prefill exchange
size_t rib_tp_prefill_buffer_bytes(int world, int rows_cap, int hidden) {
  if (world < 1 || world > RIB_TP_MAX_RANKS || rows_cap < 1 || hidden < 256 || hidden > 2048 || hidden % 256 ||
      (hidden / 256) & (hidden / 256 - 1))
    return 0;
  return round256(rib::tpp::buffer_bytes(world, rows_cap, hidden));
}

// Checks a rib_tp_prefill_exchange against M rows.
static int tpp_check(const rib_tp_prefill_exchange *ex, int M) {
  if (!ex || rib_tp_prefill_buffer_bytes(ex->world, ex->rows_cap, ex->hidden) == 0 || ex->rank < 0 ||
      ex->rank >= ex->world || M < 1 || M > ex->rows_cap)
    return RIB_EINVAL;
  for (int q = 0; q < ex->world; ++q) {
    if (!ex->buf[q]) return RIB_EINVAL;
    if (ex->buf[q] & 255u) return RIB_EALIGN;
  }
  return RIB_OK;
}

int rib_gemm_tp_partial(const void *A, int M, int K, const void *W, const rib_tp_prefill_exchange *ex,
                        void *stream) {
  using namespace rib::gemm;
  const int st = tpp_check(ex, M);
  if (st != RIB_OK) return st;
  Params p = {};
  const int H = ex->hidden;
  p.ldc = H;
  p.rpo = rib::tpp::rows_per_owner(M, ex->world);
  p.rank = ex->rank;
  p.slot_floats = static_cast<long long>(rib::tpp::rows_per_owner(ex->rows_cap, ex->world)) * H;
  for (int q = 0; q < ex->world; ++q)
    p.owner_recv[q] = reinterpret_cast<float *>(ex->buf[q] + rib::tpp::kRecvOffset);
  return gemm_run(A, M, K, W, H, kF32Owner, 256, p, stream);
}

// At most one CTA per SM, so every CTA of the grid is resident while they
// wait for one another.
extern "C++" {
template <int C>
static int tpp_reduce_launch(const rib::tpp::ReduceParams &p, cudaStream_t s) {
  constexpr int nt = rib::tpp::threads_for<C>();
  const dim3 grid(std::max(1, std::min(ceil_div(p.M, nt / 32), sm_count())));
  return launch_pdl("tp_reduce_add_rms_kernel launch", rib::tpp::tp_reduce_add_rms_kernel<C>, grid, dim3(nt), 0, s,
                    p);
}
}

int rib_tp_reduce_add_rms(const rib_tp_prefill_exchange *ex, int M, unsigned long long epoch, void *residual,
                          const void *norm_w, void *out, void *stream) {
  using namespace rib::tpp;
  const int st = tpp_check(ex, M);
  if (st != RIB_OK) return st;
  if (!residual || epoch == 0 || (norm_w && !out)) return RIB_EINVAL;
  if (!aligned16(residual) || (norm_w && (!aligned16(norm_w) || !aligned16(out)))) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  ReduceParams p = {};
  const int H = ex->hidden;
  const size_t goff = gather_offset(ex->world, ex->rows_cap, H);
  for (int q = 0; q < ex->world; ++q) {
    p.flags[q] = reinterpret_cast<unsigned long long *>(ex->buf[q] + kFlagsOffset);
    p.gather[q] = reinterpret_cast<uint16_t *>(ex->buf[q] + goff);
  }
  const uintptr_t own = static_cast<uintptr_t>(ex->buf[ex->rank]);
  p.recv = reinterpret_cast<const float *>(own + kRecvOffset);
  p.counter = reinterpret_cast<int *>(own + kCounterOffset);
  p.epoch = epoch;
  p.slot_floats = static_cast<long long>(rows_per_owner(ex->rows_cap, ex->world)) * H;
  p.world = ex->world;
  p.rank = ex->rank;
  p.M = M;
  p.H = H;
  p.rpo = rows_per_owner(M, ex->world);
  p.residual = static_cast<uint16_t *>(residual);
  p.w = static_cast<const uint16_t *>(norm_w);
  p.out = static_cast<uint16_t *>(out);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (H) {
    case 256: return tpp_reduce_launch<1>(p, s);
    case 512: return tpp_reduce_launch<2>(p, s);
    case 1024: return tpp_reduce_launch<4>(p, s);
    default: return tpp_reduce_launch<8>(p, s);
  }
}

// add_rms / rms_norm launch: warp per row for the common widths, else CTA per row.
static int row_norm_launch(const rib::model::RowParams &p, cudaStream_t st, const char *what) {
  using namespace rib::model;
  const dim3 g8(ceil_div(p.rows, 8)), b8(256);
  switch (p.W) {
    case 1024: return launch_pdl(what, add_rms_rows_kernel<4>, g8, b8, 0, st, p);
    case 2048: return launch_pdl(what, add_rms_rows_kernel<8>, g8, b8, 0, st, p);
    default:
      return launch_pdl(what, add_rms_kernel, dim3(p.rows), dim3(128), p.W * sizeof(float), st, p);
  }
}

int rib_add_rms(const void *a, const void *b, const void *w, int rows, int W, void *residual,
                void *normalized, void *stream) {
  if (!a || !b || !w || !residual || !normalized || rows < 1 || W < 8 || W % 8 || W > rib::model::kMaxK)
    return RIB_EINVAL;
  if (!aligned16(a) || !aligned16(b) || !aligned16(w) || !aligned16(residual) || !aligned16(normalized))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  rib::model::RowParams p = {static_cast<const uint16_t *>(a), static_cast<const uint16_t *>(b),
                             static_cast<const uint16_t *>(w), static_cast<uint16_t *>(residual),
                             static_cast<uint16_t *>(normalized), rows, W};
  return row_norm_launch(p, static_cast<cudaStream_t>(stream), "add_rms launch");
}

int rib_rms_norm(const void *x, const void *w, int rows, int W, void *out, void *stream) {
  if (!x || !w || !out || rows < 1 || W < 8 || W % 8 || W > rib::model::kMaxK) return RIB_EINVAL;
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  rib::model::RowParams p = {static_cast<const uint16_t *>(x), nullptr, static_cast<const uint16_t *>(w),
                             nullptr, static_cast<uint16_t *>(out), rows, W};
  return row_norm_launch(p, static_cast<cudaStream_t>(stream), "rms_norm launch");
}

int rib_swiglu(const void *gu, int rows, int F, void *out, void *stream) {
  if (!gu || !out || rows < 1 || F < 8 || F % 8) return RIB_EINVAL;
  if (!aligned16(gu) || !aligned16(out)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const long long vec = static_cast<long long>(rows) * (F / 8);
  const int grid = static_cast<int>(std::min<long long>(ceil_div(vec, 256), 16LL * sm_count()));
  return launch_pdl("swiglu_kernel launch", rib::model::swiglu_kernel, dim3(grid), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const uint16_t *>(gu), rows, F,
                    static_cast<uint16_t *>(out));
}

int rib_embed(const void *table, int vocab, int hidden, const int32_t *tokens, int n, void *out,
              void *stream) {
  if (!table || !tokens || !out || vocab < 1 || hidden < 8 || hidden % 8 || n < 1) return RIB_EINVAL;
  if (!aligned16(table) || !aligned16(out) || (reinterpret_cast<uintptr_t>(tokens) & 3u)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  return launch_pdl("embed_kernel launch", rib::model::embed_kernel, dim3(n), dim3(128), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const uint16_t *>(table), vocab, hidden,
                    tokens, static_cast<uint16_t *>(out));
}

size_t rib_argmax_workspace_bytes(void) { return 256; }

int rib_argmax_f32(const float *x, int n, int32_t *out, void *workspace, void *stream) {
  if (!x || !out || !workspace || n < 1) return RIB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15u))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(rib::model::ArgmaxWs), st);
  if (e != cudaSuccess) return rib::host_fail_cuda("cudaMemsetAsync(argmax workspace)", e);
  const int grid = std::max(1, std::min(ceil_div(n, 1024 * 4), sm_count()));
  return launch_pdl("argmax_kernel launch", rib::model::argmax_kernel, dim3(grid), dim3(1024), 0, st, x, n,
                    static_cast<rib::model::ArgmaxWs *>(workspace), out);
}


// ------------------------------------------------------------------ persistent decode step
size_t rib_qwen3_step_workspace_bytes(const rib_qwen3_model *model, int cap) {
  if (!step_model_ok(model) || cap < 1) return 0;
  return step_layout(model, cap).total;
}

int rib_qwen3_step_workspace_init(void *workspace, size_t workspace_bytes, void *stream) {
  const size_t head = kCounterRegionBytes + round256(sizeof(rib::step::Sync));
  if (!workspace || workspace_bytes < head) return RIB_EINVAL;
  if (reinterpret_cast<uintptr_t>(workspace) & 255u) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const cudaError_t e = cudaMemsetAsync(workspace, 0, head, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? RIB_OK : rib::host_fail_cuda("cudaMemsetAsync(decode step workspace init)", e);
}

int rib_qwen3_decode_step(const rib_qwen3_model *m, const uint64_t *cache_ptrs, int cap, int32_t *token,
                          int32_t *pos, int32_t *nkeys, float *logits, void *workspace, size_t workspace_bytes,
                          void *stream) {
  if (!step_model_ok(m) || !cache_ptrs || !token || !pos || !nkeys || !workspace || cap < 1) return RIB_EINVAL;
  const StepLayout lay = step_layout(m, cap);
  // split counters, the finalised-unit counter and the merge-group counters in the fixed region
  if ((static_cast<size_t>(m->num_kv_heads) * (1 + lay.g.max_groups) + 1) * sizeof(int) > kCounterRegionBytes ||
      lay.g.max_groups > rib::decode::kMergeSplits)
    return RIB_EINVAL;
  if (workspace_bytes < lay.total) return RIB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) || (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u) ||
      (reinterpret_cast<uintptr_t>(token) & 3u) || (reinterpret_cast<uintptr_t>(pos) & 3u) ||
      (reinterpret_cast<uintptr_t>(nkeys) & 3u) || (logits && (reinterpret_cast<uintptr_t>(logits) & 3u)) ||
      !aligned16(m->embed) || !aligned16(m->final_norm))
    return RIB_EALIGN;
  rib::step::Params p;
  p.L = m->num_layers;
  p.hidden = m->hidden;
  p.nq = m->num_heads;
  p.nkv = m->num_kv_heads;
  p.inter = m->intermediate;
  p.vocab = m->vocab;
  p.cap = cap;
  p.embed = static_cast<const uint16_t *>(m->embed);
  p.final_norm = static_cast<const uint16_t *>(m->final_norm);
  for (int l = 0; l < m->num_layers; ++l) {
    const rib_qwen3_layer &w = m->layers[l];
    const void *ptrs[8] = {w.qkv, w.o, w.gu, w.down, w.in_norm, w.post_norm, w.q_norm, w.k_norm};
    for (const void *q : ptrs) {
      if (!q) return RIB_EINVAL;
      if (!aligned16(q)) return RIB_EALIGN;
    }
    p.layer[l] = {static_cast<const uint16_t *>(w.qkv), static_cast<const uint16_t *>(w.o),
                  static_cast<const uint16_t *>(w.gu), static_cast<const uint16_t *>(w.down),
                  static_cast<const uint16_t *>(w.in_norm), static_cast<const uint16_t *>(w.post_norm),
                  static_cast<const uint16_t *>(w.q_norm), static_cast<const uint16_t *>(w.k_norm)};
  }
  rib::rope::rope_inv_freq(p.inv_freq, m->rope_theta);
  p.cache_ptrs = cache_ptrs;
  p.tok = token;
  p.pos = pos;
  p.nkeys = nkeys;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  for (int i = 0; i < 3; ++i) p.h[i] = reinterpret_cast<uint16_t *>(ws + lay.h_off[i]);
  p.qkv = reinterpret_cast<uint16_t *>(ws + lay.qkv_off);
  p.q = reinterpret_cast<uint16_t *>(ws + lay.q_off);
  p.o = reinterpret_cast<uint16_t *>(ws + lay.ao_off);
  p.a = reinterpret_cast<uint16_t *>(ws + lay.a_off);
  p.logits = logits;
  p.sync = reinterpret_cast<rib::step::Sync *>(ws + lay.sync_off);
  rib::decode::Params &dp = p.dp;
  dp = rib::decode::Params{};
  dp.q = p.q;
  dp.cache_ptrs = cache_ptrs;
  dp.cache = nullptr;
  dp.lens = nkeys;
  dp.n_single = 0;
  dp.max_n = cap;
  dp.cap = cap;
  dp.nq = m->num_heads;
  dp.nkv = m->num_kv_heads;
  dp.chunk = lay.g.chunk;
  dp.max_splits = lay.g.max_splits;
  dp.qscale = (1.0f / std::sqrt(128.0f)) * 1.4426950408889634f;
  dp.out = p.o;
  dp.part_ml = reinterpret_cast<float *>(ws + lay.ml_off);
  dp.part_o = reinterpret_cast<float *>(ws + lay.po_off);
  dp.counters = reinterpret_cast<int *>(ws);
  dp.world = 0;
  dp.done = dp.counters + m->num_kv_heads;
  dp.gcounters = dp.done + 1;
  dp.max_groups = lay.g.max_groups;
  dp.total_units = m->num_kv_heads;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (m->hidden == 1024 && m->num_heads * 128 == 2048 && m->intermediate == 3072)
    return step_launch<4, 8, 12, 4, 1, 3, 1>(p, 0, st);  // Qwen3-0.6B widths
  return step_launch<0, 0, 0, 0, 0, 0, 0>(p, 1, st);
}


// ------------------------------------------------------------------ batched ragged decode
int rib_decode_attention_ragged(const void *q, const uint64_t *cache_ptrs, const int32_t *caps,
                                const int32_t *lens, int batch, int max_n, int nq, int nkv, float scale,
                                void *out, void *workspace, size_t workspace_bytes, void *stream) {
  if (!q || !cache_ptrs || !caps || !lens || !out) return RIB_EINVAL;
  if (batch < 1 || nkv < 1 || nq != 2 * nkv || max_n < 1 || !(scale > 0.f)) return RIB_EINVAL;
  if (!aligned16(q) || !aligned16(out) || (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u) ||
      (reinterpret_cast<uintptr_t>(caps) & 3u) || (reinterpret_cast<uintptr_t>(lens) & 3u))
    return RIB_EALIGN;
  rib::decode::Params p = {};
  p.q = static_cast<const uint16_t *>(q);
  p.cache_ptrs = cache_ptrs;
  p.caps = caps;
  p.lens = lens;
  p.cap = max_n;  // per-sequence capacities come from caps[]
  p.nq = nq;
  p.nkv = nkv;
  p.qscale = scale * 1.4426950408889634f;
  p.out = static_cast<uint16_t *>(out);
  return decode_launch(p, batch, max_n, workspace, workspace_bytes, stream);
}

int rib_qk_norm_rope_append_batched(const void *qkv, const void *qw, const void *kw, const int32_t *pos,
                                    const uint64_t *cache_ptrs, const int32_t *caps, int batch, int nq,
                                    int nkv, double base, void *q_out, void *stream) {
  if (!qkv || !qw || !kw || !pos || !cache_ptrs || !caps || !q_out) return RIB_EINVAL;
  if (batch < 1 || nq < 1 || nkv < 1 || nq + 2 * nkv > rib::rope::kMaxItems || !(base > 0.0)) return RIB_EINVAL;
  if (!aligned16(qkv) || !aligned16(qw) || !aligned16(kw) || !aligned16(q_out) ||
      (reinterpret_cast<uintptr_t>(pos) & 3u) || (reinterpret_cast<uintptr_t>(caps) & 3u) ||
      (reinterpret_cast<uintptr_t>(cache_ptrs) & 7u))
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  rib::rope::BatchParams p;
  p.qkv = static_cast<const uint16_t *>(qkv);
  p.qw = static_cast<const uint16_t *>(qw);
  p.kw = static_cast<const uint16_t *>(kw);
  p.q_out = static_cast<uint16_t *>(q_out);
  p.cache_ptrs = cache_ptrs;
  p.caps = caps;
  p.pos = pos;
  p.nq = nq;
  p.nkv = nkv;
  rib::rope::rope_inv_freq(p.inv_freq, base);
  const int threads = ((nq + 2 * nkv + 1) / 2) * 32;
  return launch_pdl("qk_norm_rope_batched_kernel launch", rib::rope::qk_norm_rope_batched_kernel, dim3(batch),
                    dim3(threads), 0, static_cast<cudaStream_t>(stream), p);
}

int rib_gemm(const void *A, int M, int K, const void *W, int N, int epi, void *C, long long ldc,
             void *stream) {
  using namespace rib::gemm;
  if (!C || (epi != RIB_GEMM_BF16 && epi != RIB_GEMM_F32 && epi != RIB_GEMM_SWIGLU)) return RIB_EINVAL;
  Params p = {};
  p.c = C;
  p.ldc = ldc;
  int bn;
  if (epi == RIB_GEMM_SWIGLU) {
    if (N % 256 || ldc < N / 2) return RIB_EINVAL;
    bn = 256;
    p.swiglu_f = N / 2;
  } else {
    if (ldc < N || N % 8) return RIB_EINVAL;
    bn = N % 256 == 0 ? 256 : 128;  // a last tile past N is computed and not stored
  }
  if (!aligned16(C) || (ldc * (epi == RIB_GEMM_F32 ? 4 : 2)) % 16) return RIB_EALIGN;
  const int e = epi == RIB_GEMM_BF16 ? kBF16 : epi == RIB_GEMM_F32 ? kF32 : kSwiGLU;
  return gemm_run(A, M, K, W, N, e, bn, p, stream);
}

// Few-row GEMM: weight row tiles x K splits, enough CTAs to cover the SMs.
struct SmallGeom {
  int row_tiles, splits, kps;
};
SmallGeom small_geometry(int N, int K) {
  SmallGeom g;
  const int kb = K / rib::gemm::BK;
  g.row_tiles = N / rib::gemm::BM;
  const int want = std::max(1, std::min(kb, ceil_div(sm_count(), g.row_tiles)));
  g.kps = ceil_div(kb, want);
  g.splits = ceil_div(kb, g.kps);
  return g;
}

bool g_gemm_small_smem_done[kMaxDevices];

size_t rib_gemm_small_workspace_bytes(int M, int N, int K) {
  if (M < 1 || M > rib::gemm::kSmallTok || N < 128 || N % 128 || K < 64 || K % 64) return 0;
  const SmallGeom g = small_geometry(N, K);
  return static_cast<size_t>(g.splits) * N * rib::gemm::kSmallTok * sizeof(float);
}

int rib_gemm_small(const void *A, int M, int K, const void *W, int N, int epi, void *C, long long ldc,
                   void *workspace, size_t workspace_bytes, void *stream) {
  using namespace rib::gemm;
  if (!A || !W || !C || !workspace) return RIB_EINVAL;
  if (M < 1 || M > kSmallTok || N < 128 || N % 128 || K < 64 || K % 64) return RIB_EINVAL;
  if (epi != RIB_GEMM_BF16 && epi != RIB_GEMM_SWIGLU) return RIB_EINVAL;
  const int n_out = epi == RIB_GEMM_SWIGLU ? N / 2 : N;
  if (n_out % kReduceCols || ldc < n_out) return RIB_EINVAL;
  if (workspace_bytes < rib_gemm_small_workspace_bytes(M, N, K)) return RIB_EINVAL;
  if (!aligned16(A) || !aligned16(W) || !aligned16(C) || !aligned16(workspace) || (ldc * 2) % 16)
    return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  const SmallGeom g = small_geometry(N, K);
  SmallParams p = {};
  if (!gemm_map(&p.tm_w, W, N, K, K, BM) || !gemm_map(&p.tm_x, A, M, K, K, kSmallTok)) return RIB_ECUDA;
  p.M = M;
  p.N = N;
  p.K = K;
  p.kps = g.kps;
  p.part = static_cast<float *>(workspace);
  const int smem = static_cast<int>(sizeof(SmallSmem)) + 1024;
  if (!set_smem_once(gemm_small_kernel, smem, g_gemm_small_smem_done))
    return rib::host_fail(RIB_ECUDA, "cudaFuncSetAttribute(gemm small smem)", smem);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rc = launch_pdl("gemm_small_kernel launch", gemm_small_kernel, dim3(g.row_tiles, g.splits),
                            dim3(NTHREADS), smem, st, p);
  if (rc != RIB_OK) return rc;
  SmallReduceParams r = {};
  r.part = p.part;
  r.splits = g.splits;
  r.N = N;
  r.M = M;
  r.swiglu_f = epi == RIB_GEMM_SWIGLU ? N / 2 : 0;
  r.c = static_cast<uint16_t *>(C);
  r.ldc = ldc;
  return launch_pdl("gemm_small_reduce_kernel launch", gemm_small_reduce_kernel, dim3(n_out / kReduceCols),
                    dim3(256), 0, st, r);
}

int rib_rope_table(int pos0, int count, double base, void *table, void *stream) {
  if (!table || pos0 < 0 || count < 1 || !(base > 0.0)) return RIB_EINVAL;
  if (!aligned16(table)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  rib::rope::Params rp = {};
  rib::rope::rope_inv_freq(rp.inv_freq, base);
  return launch_pdl("rope_table_kernel launch", rib::gemm::rope_table_kernel, dim3(count), dim3(64), 0,
                    static_cast<cudaStream_t>(stream), pos0, count, rp, static_cast<float2 *>(table));
}

int rib_gemm_qkv_rope(const void *A, int M, int K, const void *W, int nq, int nkv, const void *qw,
                      const void *kw, const void *rope_table, int pos0, void *q_out, int Lp, void *cache,
                      int cap, void *stream) {
  using namespace rib::gemm;
  if (!qw || !kw || !rope_table || !q_out || !cache || nq < 1 || nkv < 1 || pos0 < 0 || Lp < M || cap < 1)
    return RIB_EINVAL;
  if (static_cast<long long>(pos0) + M > cap) return RIB_ECAPACITY;
  if (!aligned16(qw) || !aligned16(kw) || !aligned16(rope_table) || !aligned16(q_out) || !aligned16(cache))
    return RIB_EALIGN;
  Params p = {};
  p.qw = static_cast<const uint16_t *>(qw);
  p.kw = static_cast<const uint16_t *>(kw);
  p.rope = static_cast<const float2 *>(rope_table);
  p.pos0 = pos0;
  p.nq = nq;
  p.nkv = nkv;
  p.q_out = static_cast<uint16_t *>(q_out);
  p.Lp = Lp;
  p.cache = static_cast<uint16_t *>(cache);
  p.cap = cap;
  // tiles of 128 rows cover Lp (Q pad rows are written as zero)
  // two heads per 256-wide tile ((nq + 2 nkv) = 4 nkv heads: always even)
  const int status = gemm_run(A, M, K, W, (nq + 2 * nkv) * 128, kQKRope, 256, p, stream);
  return status;
}

int rib_argmax_rows_f32(const float *x, int rows, int n, int32_t *out, void *stream) {
  if (!x || !out || rows < 1 || n < 1) return RIB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u)) return RIB_EALIGN;
  if (!bind_stream_device(stream)) return rib::host_fail(RIB_ECUDA, "bind stream device", 0);
  return launch_pdl("argmax_rows_kernel launch", rib::model::argmax_rows_kernel, dim3(rows), dim3(1024), 0,
                    static_cast<cudaStream_t>(stream), x, n, out);
}

}  // extern "C"
