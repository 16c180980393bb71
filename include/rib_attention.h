/*
 * rib_attention.h -- C ABI of the B200 (sm_100a) Qwen3 attention hot path.
 *
 * The reference (aeilot/roofline-inference, agent-test/v2) runs this path as
 * Metal kernels compiled by MLX plus one MLX library call.  Each entry point
 * below replaces one of those interfaces; the citation names the reference
 * function whose arguments and results it keeps.
 *
 * Conventions (all entry points):
 *   - Pointers are DEVICE pointers unless the name ends in `_host`.  Tensors
 *     are BF16 stored as uint16 bit patterns, row-major and contiguous in the
 *     layout stated per argument.  The caller owns every buffer; the library
 *     never allocates or frees on these paths and keeps no per-call state.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call
 *     only enqueues work (kernels, and for decode a small memset of its
 *     counters) and returns; none synchronises.
 *   - Return value: RIB_OK (0) or one of the RIB_E* codes below.  Argument
 *     checks run on the host before anything is launched, so an error return
 *     means nothing was enqueued.
 *   - head_dim is 128 and the GQA group is 2 (n_q_heads == 2 * n_kv_heads),
 *     the same preconditions as the reference engine
 *     (agent-test/v2/engine.py:69-70, agent-test/v2/attention.py:181).
 */
#ifndef RIB_ATTENTION_H
#define RIB_ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The Python layer maps 1-3 to ValueError and 4-5 to
 * RuntimeError, matching the reference's ValueError on shape/capacity errors
 * (agent-test/v2/engine.py:45-46, 69-70). */
#define RIB_OK 0
#define RIB_EINVAL 1    /* bad shape / argument                         */
#define RIB_ECAPACITY 2 /* "KV capacity exceeded" (engine.py:45-46)     */
#define RIB_EALIGN 3    /* pointer not 16-byte aligned                  */
#define RIB_ECUDA 4     /* a CUDA runtime call failed                   */
#define RIB_ETIMEOUT 5  /* a device-side wait gave up (bounded spin)    */

/* Library version, (major << 16) | minor. */
int rib_version(void);

/* Human-readable text for a status code (static storage). */
const char *rib_status_string(int status);

/* Text of the last host-side failure on the calling thread (which step and
 * which CUDA error), "" if none yet.  Static thread-local storage. */
const char *rib_last_error_string(void);

/* Reads and clears the device-side status word of the current device: 0 if
 * no kernel recorded a timeout since the last call, RIB_ETIMEOUT otherwise.
 * Synchronises the current device. */
int rib_take_device_status(int *status_host);

/* Wall-clock limit of every device-side wait of this library (mbarrier
 * waits, the NVLink gather's epoch poll, the tensor-parallel word polls, the
 * persistent step's grid barrier) on the current device, in nanoseconds:
 * 2 s unless set, accepted range 1 ms .. 60 s (RIB_EINVAL otherwise).  A wait
 * that runs out records RIB_ETIMEOUT (rib_take_device_status) and its kernel
 * returns instead of spinning; the reference's analogue is the v3 harness's
 * per-unit timeout with an exclusion record (agent-test/v3/run.py:238-261).
 * The new limit applies to kernels launched after the call returns; set it
 * while none of this library's kernels runs on the device.  No reference
 * counterpart as an entry point. */
int rib_set_wait_limit_ns(unsigned long long ns);
int rib_get_wait_limit_ns(unsigned long long *ns);

/* ------------------------------------------------------------------------ *
 * Fused per-head RMSNorm + RoPE, one token (decode).
 * Replaces qk_norm_rope(qkv, qw, kw, pos, nq, nkv, base)
 *   (agent-test/v2/kernels.py:157-164, Metal source kernels.py:116-146).
 *   qkv    [(nq + 2*nkv) * 128]   q heads, then k heads, then v heads
 *   qw, kw [128]                  RMSNorm weights for q and k
 *   pos                           RoPE position (the reference passes it as a
 *                                 1-element int32 array; here by value)
 *   q_out  [nq, 128]              == the reference's q [1, nq, 1, 128]
 *   kv_out [2, nkv, 128]          == the reference's kv [2, nkv, 1, 128]
 * RMSNorm eps is 1e-6; rounding points n = bf16(w * bf16(x * inv)); RoPE is
 * the non-traditional form pairing (d, d+64) with theta = pos * base^(-d/64),
 * formed in FP32 as the reference forms it (float(pos) * exp2(-(d/64) *
 * log2(base)), kernels.py:134-138) and evaluated to full accuracy.
 * V is copied bit for bit.
 * ------------------------------------------------------------------------ */
int rib_qk_norm_rope(const void *qkv, const void *qw, const void *kw, int pos,
                     int nq, int nkv, double base, void *q_out, void *kv_out,
                     void *stream);

/* ------------------------------------------------------------------------ *
 * Fused RMSNorm + RoPE for L tokens at positions offset .. offset+L-1.
 * Replaces qk_norm_rope_prefill(qkv, qw, kw, offset, nq, nkv, base, Lp)
 *   (agent-test/v2/kernels.py:215-224, Metal source kernels.py:169-204).
 *   qkv    [L, (nq + 2*nkv) * 128]
 *   q_out  [nq, Lp, 128]   rows L..Lp-1 are written as zeros (the reference
 *                          launches with init_value=0, kernels.py:223)
 *   kv_out [2, nkv, L, 128]
 * Requires Lp >= L.
 * ------------------------------------------------------------------------ */
int rib_qk_norm_rope_prefill(const void *qkv, int L, const void *qw,
                             const void *kw, int offset, int nq, int nkv,
                             double base, int Lp, void *q_out, void *kv_out,
                             void *stream);

/* ------------------------------------------------------------------------ *
 * The same kernel with the KV-cache write fused in: K (normed + roped) and V
 * go straight to rows offset .. offset+L-1 of one layer's cache.
 * Replaces the pair qk_norm_rope[_prefill] (kernels.py:157/215) followed by
 * Cache.update (agent-test/v2/engine.py:42-48), called at engine.py:111-113
 * and engine.py:152-153.
 *   cache  [2, nkv, cap, 128]   one layer of Cache.kv (engine.py:38)
 *   q_out  [nq, Lp, 128]        (Lp == 1 for a decode token)
 * Returns RIB_ECAPACITY if offset + L > cap, as Cache.update raises
 * ValueError("KV capacity exceeded") (engine.py:45-46).
 * ------------------------------------------------------------------------ */
int rib_qk_norm_rope_append(const void *qkv, int L, const void *qw,
                            const void *kw, int offset, int nq, int nkv,
                            double base, int Lp, void *q_out, void *cache,
                            int cap, void *stream);

/* ------------------------------------------------------------------------ *
 * GQA decode attention: one query token per sequence against n cached keys.
 * Replaces mx.fast.scaled_dot_product_attention(q, K, V, scale) as called by
 * Engine.decode (agent-test/v2/engine.py:154-155), where K, V are the views
 * cache.views(i, n) == buf[0:1, :, :n], buf[1:2, :, :n] (engine.py:50-52).
 *   q      [nq, 128]             post-RoPE query (the reference's [1,nq,1,128])
 *   cache  [2, nkv, cap, 128]    one layer of the KV cache
 *   n      number of valid keys (offset + 1 in Engine.decode, engine.py:149)
 *   out    [nq, 128]             == [1, nq, 1, 128], o_proj input layout
 *   workspace / workspace_bytes  device scratch of at least
 *          rib_decode_workspace_bytes(1, n, nkv) bytes.  Its first 16 KiB
 *          hold split counters that must be zero before the workspace's
 *          first use (allocate it zero-filled or call
 *          rib_decode_workspace_init once); every completed call leaves them
 *          zero again, so calls of any shape can share one workspace and no
 *          call enqueues a memset (except launches of more than 4095
 *          sequence x KV-head units, which clear a larger region
 *          themselves).  After a call whose launch reported RIB_ETIMEOUT
 *          through rib_take_device_status, initialise it again.  Calls that
 *          share a workspace must not overlap on the device.
 * Softmax and accumulation in FP32; output rounded to BF16 once.
 * ------------------------------------------------------------------------ */
size_t rib_decode_workspace_bytes(int batch, int max_n, int nkv);

/* Which decode kernel rib_decode_attention / _batched / _ragged / _gather
 * launch for `batch` sequences of at most max_n keys over nkv KV heads on
 * the current device: 0 the fixed-split kernel (decode_kernel), 1 the
 * stream-K kernel (decode_streamk_kernel), -RIB_EINVAL for a bad size.
 * (rib_decode_attention_qkv and the no-allocation entry point always take
 * the split kernel.)  For reporting and profiling; no call needs it. */
int rib_decode_kernel_choice(int batch, int max_n, int nkv);

/* Zeroes the counter region of a decode workspace (an enqueued memset on
 * `stream`); workspace_bytes >= 16384. */
int rib_decode_workspace_init(void *workspace, size_t workspace_bytes,
                              void *stream);

int rib_decode_attention(const void *q, const void *cache, int cap, int n,
                         int nq, int nkv, float scale, void *out,
                         void *workspace, size_t workspace_bytes,
                         void *stream);

/* ------------------------------------------------------------------------ *
 * Decode attention that allocates nothing (no counterpart in the reference).
 * Same arguments and results as rib_decode_attention, minus the workspace:
 * its scratch is a fixed 2 MiB array inside this library's device memory.
 * For callers that cannot call cudaMalloc or hand over device scratch (a
 * host whose device memory is owned by another allocator or a hard memory
 * budget, a binding with no device allocator of its own).
 *   - Sizes whose scratch (rib_decode_workspace_bytes(1, n, nkv)) exceeds
 *     2 MiB are rejected with RIB_EINVAL (every n <= 909312 fits at 8 KV heads).
 *   - The first call on a device looks up the array's device address; make
 *     that first call before any stream capture.
 *   - The array starts zeroed and every call leaves its counters zero, so
 *     calls need no memset; calls that overlap on the GPU (other streams,
 *     other threads) race.
 * ------------------------------------------------------------------------ */
int rib_decode_attention_noalloc(const void *q, const void *cache, int cap,
                                 int n, int nq, int nkv, float scale,
                                 void *out, void *stream);

/* ------------------------------------------------------------------------ *
 * Batched ragged decode: B independent sequences, each with its own
 * contiguous per-sequence cache and its own length.  Generalises the
 * single-sequence call above (the reference is batch 1 only, README.md
 * "Single stream"; engine.py:33-40 is the per-sequence cache it generalises).
 *   q          [B, nq, 128]
 *   cache_ptrs device array of B pointers, each to a [2, nkv, cap, 128] cache
 *   lens       device array of B int32 key counts (1 <= lens[b] <= cap)
 *   max_n      host upper bound on lens[] (sizes the launch)
 *   out        [B, nq, 128]
 *   workspace  at least rib_decode_workspace_bytes(B, max_n, nkv) bytes,
 *              same contract as above.
 * ------------------------------------------------------------------------ */
int rib_decode_attention_batched(const void *q, const uint64_t *cache_ptrs,
                                 const int32_t *lens, int batch, int max_n,
                                 int cap, int nq, int nkv, float scale,
                                 void *out, void *workspace,
                                 size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ *
 * Decode attention fused with the all-gather of head outputs over NVLink.
 * The KV heads of a model are sharded over the ranks of one node (rank r of
 * `world` owns nkv = 8/world of them and query heads 2h, 2h+1); this call
 * runs the batched decode above for the local heads and stores each finished
 * output straight into every rank's gathered buffer (peer stores through
 * CUDA IPC mappings), then exchanges an epoch flag with every peer.  When it
 * completes on `stream`, this rank's buffer holds all ranks' outputs.  It
 * replaces the decode SDPA (engine.py:155) plus the NCCL all-gather a
 * head-sharded engine would need (the reference is single-GPU).
 *   Gathered layout: region (epoch & 1) of each buffer,
 *     [batch][world * nq][128] BF16, rank r's heads at [r*nq, (r+1)*nq).
 *   Signal slots: 8 uint64 after the two regions; slot s holds the last
 *     epoch rank s published.  Buffers start zeroed.
 *   epoch: 1 for the first call, +1 per call, the same on every rank.
 * Every rank must make the call with the same epoch; a rank that does not
 * arrive within 2 s makes the others record RIB_ETIMEOUT and return.
 * Setup: rib_peer_buffer_alloc on each rank, exchange the 64-byte IPC
 * handles (e.g. torch.distributed all_gather_object), rib_peer_buffer_open
 * the peers' handles; tear down with rib_peer_buffer_close / _free.
 * ------------------------------------------------------------------------ */
#define RIB_MAX_PEERS 8

typedef struct rib_peer_gather {
  int world;                       /* ranks in the gather, 1..8             */
  int rank;                        /* this rank                             */
  uint64_t out[RIB_MAX_PEERS];     /* per rank: buffer base, as mapped here */
  uint64_t sig[RIB_MAX_PEERS];     /* per rank: address of its signal slots */
  size_t region_bytes;             /* bytes of one output region            */
} rib_peer_gather;

size_t rib_peer_buffer_bytes(int batch, int nq_total);
int rib_peer_buffer_alloc(int device, size_t bytes, void **dev_ptr,
                          void *ipc_handle /* 64 bytes out */);
int rib_peer_buffer_open(int device, const void *ipc_handle, void **peer_ptr);
int rib_peer_buffer_close(int device, void *peer_ptr);
int rib_peer_buffer_free(int device, void *dev_ptr);

/* Host-epoch form.  lens, cache_ptrs and every cache row below lens[b] - 1
 * must be complete when the launch starts (written by host copies, by a
 * kernel that does not trigger programmatic launch, or earlier): each CTA
 * streams its first K/V tiles before waiting for the previous kernel, so a
 * call overlaps the previous call's exchange with the peers.  q and the new
 * token's row may come from the kernel launched just before. */
int rib_decode_attention_gather(const void *q, const uint64_t *cache_ptrs,
                                const int32_t *lens, int batch, int max_n,
                                int cap, int nq, int nkv, float scale,
                                const rib_peer_gather *g,
                                unsigned long long epoch, void *workspace,
                                size_t workspace_bytes, void *stream);

/* The same with the epoch kept on the device, for CUDA-graph replay: the call
 * uses *epoch_dev + 1 (an 8-byte-aligned counter in device memory, zero on
 * every rank before the first call) and stores it back, so every replay
 * gets the next epoch.  The output region alternates with the epoch as
 * above; after every rank's outputs have arrived, the kernel also copies
 * them into out_copy [batch, world * nq, 128], a fixed address that the
 * captured consumer can read.  Every rank makes the same sequence of calls
 * with its own counter. */
int rib_decode_attention_gather_dev(const void *q, const uint64_t *cache_ptrs,
                                    const int32_t *lens, int batch, int max_n,
                                    int cap, int nq, int nkv, float scale,
                                    const rib_peer_gather *g,
                                    unsigned long long *epoch_dev,
                                    void *out_copy, void *workspace,
                                    size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------ *
 * Causal GQA prefill attention (tcgen05 / TMEM flash attention).
 * Replaces attention(Q, K, V, qL, kL, scale, ...) (agent-test/v2/attention.py
 * :177-185, Metal source attention.py:18-166).
 *   Q      [H, qLp, 128]         post-RoPE queries; rows >= qL are ignored
 *   K, V   [nkv, cap, 128]       the K and V halves of one cache layer
 *                                (the reference passes buf[0:1], buf[1:2])
 *   O      [qL, H * 128]         o_proj input layout (attention.py:10)
 * Causal mask is bottom-right aligned: query i sees keys <= kL - qL + i
 * (attention.py:24, 111).  Requires H == 2 * nkv, qL <= qLp, qL <= kL <= cap.
 *   workspace  device scratch of rib_prefill_workspace_bytes(kL, nkv) bytes
 *              (16-byte aligned): the call writes an FP16 copy of V there
 *              and runs P.V in FP16 (the reference keeps P in FP32,
 *              attention.py:141-153; FP16 P keeps the error at the BF16
 *              rounding floor).  V values beyond the FP16 range (|v| > 65504)
 *              are recorded as RIB_EINVAL on the device status word.
 * ------------------------------------------------------------------------ */
size_t rib_prefill_workspace_bytes(int kL, int nkv);
int rib_prefill_attention(const void *Q, const void *K, const void *V, int qL,
                          int kL, int qLp, int cap, int H, int nkv,
                          float scale, void *O, void *workspace,
                          size_t workspace_bytes, void *stream);

/* ======================================================================== *
 * Qwen3 forward around the attention path (agent-test/v2/engine.py:102-163).
 * ======================================================================== */

/* Fused RMSNorm + RoPE + KV append with the position read on the device, so
 * a captured CUDA graph can replay a decode step at a new position.  Same as
 * rib_qk_norm_rope_append with offset = *offset_dev (an int32 in device
 * memory); the reference passes the position as an int32 array too
 * (qk_norm_rope(qkv, qw, kw, pos, ...), agent-test/v2/kernels.py:157-164).
 * offset + L > cap is detected on the device: nothing is written and the
 * device status word (rib_take_device_status) reads RIB_ECAPACITY. */
int rib_qk_norm_rope_append_dev(const void *qkv, int L, const void *qw,
                                const void *kw, const int32_t *offset_dev,
                                int nq, int nkv, double base, int Lp,
                                void *q_out, void *cache, int cap, void *stream);

/* rib_qk_norm_rope_prefill with the first position read on the device
 * (*offset_dev, int32): the form of qk_norm_rope(qkv, qw, kw, pos, ...)
 * (agent-test/v2/kernels.py:157-164), whose pos is an int32 array, and of
 * qk_norm_rope_prefill (kernels.py:215-224), without a host read of the
 * position.  L = 1, Lp = 1 is the single-token form.  Outputs as
 * rib_qk_norm_rope_prefill; a negative position writes nothing and the device
 * status word reads RIB_ECAPACITY. */
int rib_qk_norm_rope_prefill_dev(const void *qkv, int L, const void *qw,
                                 const void *kw, const int32_t *offset_dev,
                                 int nq, int nkv, double base, int Lp,
                                 void *q_out, void *kv_out, void *stream);

/* Epilogues of rib_gemv. */
#define RIB_EPI_NONE 0     /* y = bf16(W x), or FP32 W x when out_f32      */
#define RIB_EPI_RESIDUAL 1 /* y = bf16(res + bf16(W x))                    */
#define RIB_EPI_SWIGLU 2   /* W = [gate; up] (N = 2F rows), y[F]:
                              g = bf16(W_g x), u = bf16(W_u x),
                              y = bf16(bf16(g * bf16(sigmoid(g))) * u)     */

/* Launch hint OR-ed into rib_gemv's epi: 16 warps per CTA instead of 8, so
 * half as many CTAs each stage and normalise x once for twice the rows.
 * Results are identical.  It pays when the launch follows another GEMV; right
 * after a decode-attention launch the narrow form is faster (its CTAs fit
 * beside the attention's and start their weight loads before it ends).
 * Honoured for one row per warp, K in {256, 512, 768, 1024, 1536, 2048,
 * 3072}; otherwise ignored.  No counterpart in the reference. */
#define RIB_GEMV_WIDE 0x100

/* Batch-1 GEMV with fused input RMSNorm and epilogue.  Replaces
 * gemv(W, x, nw=, res=, swiglu=, out_float=) (agent-test/v2/kernels.py
 * :103-113, Metal source :19-97).
 *   W    [N, K] BF16 row-major, K a multiple of 8, K <= 8192
 *   x    [K] BF16
 *   nw   [K] RMSNorm weight or NULL; with it the kernel uses
 *        bf16(nw * bf16(x / sqrt(mean(x^2) + 1e-6))) in place of x
 *   res  [N] BF16 residual (RIB_EPI_RESIDUAL only, NULL otherwise)
 *   y    [N] BF16 ([N/2] for RIB_EPI_SWIGLU), or [N] FP32 when out_f32
 *        (RIB_EPI_NONE only: the logits, gemv(..., out_float=True)). */
int rib_gemv(const void *W, int N, int K, const void *x, const void *nw,
             const void *res, int epi, int out_f32, void *y, void *stream);

/* Residual add + RMSNorm over `rows` rows of width W (multiple of 8,
 * <= 8192).  Replaces add_rms(a, b, weight) (agent-test/v2/kernels.py
 * :262-268, Metal source :227-259): residual = bf16(a + b), normalized =
 * bf16(w * bf16(residual / sqrt(mean(residual^2) + 1e-6))). */
int rib_add_rms(const void *a, const void *b, const void *w, int rows, int W,
                void *residual, void *normalized, void *stream);

/* RMSNorm of `rows` rows: out = bf16(w * bf16(x / sqrt(mean(x^2) + 1e-6))).
 * Replaces mx.fast.rms_norm(h, w, eps) (agent-test/v2/engine.py:109, 140). */
int rib_rms_norm(const void *x, const void *w, int rows, int W, void *out,
                 void *stream);

/* SwiGLU of a fused gate/up product: gu [rows, 2F] (gate columns first) ->
 * out [rows, F] with the RIB_EPI_SWIGLU rounding.  Replaces
 * swiglu(*mx.split(x @ W_gu^T, 2, -1)) (agent-test/v2/engine.py:28-30, 133-134).
 * F is a multiple of 8. */
int rib_swiglu(const void *gu, int rows, int F, void *out, void *stream);

/* Embedding gather out[i] = table[tokens[i]] for n int32 token ids in device
 * memory.  Replaces self.embed[tokens] (agent-test/v2/engine.py:108, 147).
 * An id outside [0, vocab) writes a zero row and sets the device status
 * word to RIB_EINVAL. */
int rib_embed(const void *table, int vocab, int hidden, const int32_t *tokens,
              int n, void *out, void *stream);

/* Greedy token: out[0] = index of the largest of n FP32 logits (the first on
 * ties).  Replaces mx.argmax(logits) (agent-test/v2/engine.py:163, 183).
 * workspace: rib_argmax_workspace_bytes() bytes of device memory, 16-byte
 * aligned; cleared by the call itself, so it needs no initialisation, but
 * calls that overlap in time need separate workspaces. */
size_t rib_argmax_workspace_bytes(void);
int rib_argmax_f32(const float *x, int n, int32_t *out, void *workspace,
                   void *stream);

/* ------------------------------------------------------------------------ *
 * Whole decode step of a dense Qwen3 model in one cooperative launch: the
 * per-token loop of Engine.decode (agent-test/v2/engine.py:145-163) with the
 * same kernels' arithmetic, but one persistent kernel instead of one launch
 * per operation (no counterpart in the reference, which launches 7 kernels
 * per layer).
 *   model      weights in the engine layout (engine.py:80-88); every
 *              pointer 16-byte aligned.  head_dim 128, num_heads ==
 *              2 * num_kv_heads, hidden / intermediate / num_heads*128
 *              multiples of 256, num_heads + 2*num_kv_heads <= 64,
 *              num_layers <= 64.
 *   cache_ptrs device array [num_layers] of layer caches [2, nkv, cap, 128]
 *   token, pos, nkeys   device int32 scalars: the token to decode, its
 *              position (the cache offset) and pos + 1.  The step writes the
 *              next greedy token into *token and advances *pos and *nkeys, so
 *              calling it again decodes the following token.
 *   logits     [vocab] FP32 logits of the step, or NULL
 *   workspace  rib_qwen3_step_workspace_bytes(model, cap) bytes, 256-byte
 *              aligned, zero-filled before first use (or
 *              rib_qwen3_step_workspace_init); steps leave it ready for the
 *              next one.  After a failed step (rib_take_device_status != 0)
 *              initialise it again.
 * ------------------------------------------------------------------------ */
#define RIB_QWEN3_MAX_LAYERS 64
typedef struct rib_qwen3_layer {
  const void *qkv;        /* [(nq + 2 nkv) * 128, hidden]  q_proj; k_proj; v_proj */
  const void *o;          /* [hidden, nq * 128] */
  const void *gu;         /* [2 * intermediate, hidden]     gate_proj; up_proj */
  const void *down;       /* [hidden, intermediate] */
  const void *in_norm;    /* [hidden] */
  const void *post_norm;  /* [hidden] */
  const void *q_norm;     /* [128] */
  const void *k_norm;     /* [128] */
} rib_qwen3_layer;

typedef struct rib_qwen3_model {
  int num_layers, hidden, num_heads, num_kv_heads, intermediate, vocab;
  double rope_theta;
  const void *embed;      /* [vocab, hidden], also the LM head (tied) */
  const void *final_norm; /* [hidden] */
  rib_qwen3_layer layers[RIB_QWEN3_MAX_LAYERS];
} rib_qwen3_model;

size_t rib_qwen3_step_workspace_bytes(const rib_qwen3_model *model, int cap);
int rib_qwen3_step_workspace_init(void *workspace, size_t workspace_bytes,
                                  void *stream);
int rib_qwen3_decode_step(const rib_qwen3_model *model,
                          const uint64_t *cache_ptrs, int cap, int32_t *token,
                          int32_t *pos, int32_t *nkeys, float *logits,
                          void *workspace, size_t workspace_bytes,
                          void *stream);

/* ------------------------------------------------------------------------ *
 * Batched ragged decode of the whole model: B independent sequences, each in
 * its own contiguous cache of its own capacity (engine.py:33-40 generalised
 * to many sequences; the reference engine is single-stream).
 *
 * Decode attention over per-sequence caches: as
 * rib_decode_attention_batched, with caps[b] the capacity (rows per head)
 * of sequence b's cache [2, nkv, caps[b], 128] and max_n >= every lens[b]. */
int rib_decode_attention_ragged(const void *q, const uint64_t *cache_ptrs,
                                const int32_t *caps, const int32_t *lens,
                                int batch, int max_n, int nq, int nkv,
                                float scale, void *out, void *workspace,
                                size_t workspace_bytes, void *stream);

/* Fused RMSNorm + RoPE + KV append of one new token per sequence:
 *   qkv [B, (nq + 2 nkv) * 128], pos [B] device int32 (each token's position,
 *   the cache row written), cache_ptrs [B], caps [B] as above,
 *   q_out [B, nq, 128].
 * A position outside [0, caps[b]) writes nothing for that sequence and sets
 * the device status word to RIB_ECAPACITY. */
int rib_qk_norm_rope_append_batched(const void *qkv, const void *qw,
                                    const void *kw, const int32_t *pos,
                                    const uint64_t *cache_ptrs,
                                    const int32_t *caps, int batch, int nq,
                                    int nkv, double base, void *q_out,
                                    void *stream);

/* Decode attention with the new token's norm + RoPE + append fused in: as
 * rib_decode_attention_batched (uniform capacity cap, lens[b] keys of
 * sequence b), but q is formed inside the kernel from the token's projection
 * qkv [B, (nq + 2 nkv) * 128] (per-head RMSNorm with qw / kw, RoPE at
 * position lens[b] - 1 with base `base`), and the token's K and V rows are
 * written into the cache at that position first.  Outputs and cache rows are
 * bit-identical to rib_qk_norm_rope_append_batched followed by
 * rib_decode_attention_batched; one launch and one dependency fewer per
 * layer (agent-test/v2/engine.py:150-155 in one kernel).
 * The kernel starts streaming the cache before its programmatic-launch wait:
 * lens, cache_ptrs and the cache rows below lens[b] - 1 must be complete
 * when it starts (written by host copies, by a kernel that does not trigger
 * programmatic launch, or earlier); only qkv may come from the kernel
 * launched immediately before. */
int rib_decode_attention_qkv(const void *qkv, const void *qw, const void *kw,
                             double base, const uint64_t *cache_ptrs,
                             const int32_t *lens, int batch, int max_n, int cap,
                             int nq, int nkv, float scale, void *out,
                             void *workspace, size_t workspace_bytes,
                             void *stream);

/* ------------------------------------------------------------------------ *
 * Prefill projections: a persistent tcgen05 GEMM C = epi(A W^T) with
 * A [M][K] and W [N][K] row-major BF16 (K a multiple of 64).  Replaces the
 * matmul the reference's engine runs for prompts of more than 32 tokens
 * (agent-test/v2/engine.py:95-99; mx.matmul, a library GEMM) and fuses what
 * follows it in Engine.prefill (engine.py:110-135).
 *   RIB_GEMM_BF16    C [M][ldc] = bf16(A W^T); N a multiple of 8
 *   RIB_GEMM_F32     C [M][ldc] FP32 (tensor-parallel partial sums, logits)
 *   RIB_GEMM_SWIGLU  W = [gate; up] (N = 2F rows, F a multiple of 128);
 *                    C [M][ldc >= F] = bf16(bf16(g bf16(sigmoid g)) u),
 *                    g = bf16(A Wg^T), u = bf16(A Wu^T) (engine.py:28-30)
 * ------------------------------------------------------------------------ */
#define RIB_GEMM_BF16 0
#define RIB_GEMM_F32 1
#define RIB_GEMM_SWIGLU 2
int rib_gemm(const void *A, int M, int K, const void *W, int N, int epi,
             void *C, long long ldc, void *stream);

/* The same product for at most 64 rows of A (a batched decode step over up
 * to 64 sequences, a short prompt), where the weights are what has to
 * stream: the tcgen05 tile is 128 weight rows x 64 tokens (the operands swap
 * roles) and K is split over enough CTAs to cover the GPU, each writing an
 * FP32 partial to `workspace`; a second launch sums the partials of each
 * output in split order and applies the epilogue.  Every weight byte is read
 * once.  Replaces the reference's skinny / library GEMM for few rows
 * (agent-test/v2/kernels.py:273-334, engine.py:95-99).
 *   1 <= M <= 64, K a multiple of 64, N a multiple of 128;
 *   epi RIB_GEMM_BF16 or RIB_GEMM_SWIGLU;
 *   workspace: rib_gemm_small_workspace_bytes(M, N, K) bytes (16-byte
 *   aligned, no initial contents); calls sharing it must not overlap on the
 *   device. */
size_t rib_gemm_small_workspace_bytes(int M, int N, int K);
int rib_gemm_small(const void *A, int M, int K, const void *W, int N, int epi,
                   void *C, long long ldc, void *workspace,
                   size_t workspace_bytes, void *stream);

/* (cos, sin) FP32 pairs [count][64] of the RoPE angles of positions
 * pos0 .. pos0 + count - 1 (theta as kernels.py:134-138 forms it), the
 * table rib_gemm_qkv_rope reads.  16-byte aligned, count * 512 bytes. */
int rib_rope_table(int pos0, int count, double base, void *table, void *stream);

/* The QKV projection of M prompt tokens fused with the per-head QK-RMSNorm,
 * RoPE and KV-cache append: replaces matmul(x, qkv) -> qk_norm_rope_prefill
 * -> Cache.update (engine.py:111-113; kernels.py:169-224) without writing
 * the qkv activations.  W [(nq + 2 nkv) * 128][K] in the engine's fused
 * order (q heads, k heads, v heads); qw, kw [128]; rope_table from
 * rib_rope_table(pos0, >= M, ...).  Writes Q [nq][Lp][128] (rows [M, Lp)
 * zero) and cache rows pos0 .. pos0 + M - 1 of cache [2][nkv][cap][128]. */
int rib_gemm_qkv_rope(const void *A, int M, int K, const void *W, int nq,
                      int nkv, const void *qw, const void *kw,
                      const void *rope_table, int pos0, void *q_out, int Lp,
                      void *cache, int cap, void *stream);

/* Greedy token of each row of x [rows, n] FP32 (the first index on ties). */
int rib_argmax_rows_f32(const float *x, int rows, int n, int32_t *out,
                        void *stream);

/* ------------------------------------------------------------------------ *
 * Tensor parallelism of the decode projections over the GPUs of one node
 * (no counterpart in the single-GPU reference; it splits the GEMVs of
 * Engine.decode, agent-test/v2/engine.py:150-162, over ranks).
 *
 * Rank r holds its KV heads' rows of the QKV projection, the matching
 * columns of the O projection, a slice of the gate and up rows, the matching
 * columns of the down projection and a slice of the LM-head rows.  The O and
 * down GEMVs then give FP32 partial sums of the full hidden vector, which
 * every rank stores straight into every rank's exchange buffer over NVLink
 * (RIB_EPI_PEER_PARTIAL); the next GEMV reads its input as
 * bf16(residual + bf16(sum of the partials in rank order)), the rounding of
 * RIB_EPI_RESIDUAL, so every rank computes identical activations.
 *
 * Exchange buffer of one rank (rib_tp_buffer_bytes(world, slot) bytes,
 * zeroed, shared through rib_peer_buffer_alloc / _open): [2 regions][world]
 * [slot] 8-byte words.  Exchange number e uses region e & 1; a word holds a
 * value in its low 32 bits and the low 32 bits of e in its high 32 bits and
 * is written with one 8-byte store, so a reader polls the words themselves
 * (bounded) until they carry e: no fence and no separate flag.
 * epoch: device u64 counting this rank's exchanges (zero on every rank
 * before the first); done: device u32 arrival counter (zero; every call
 * leaves it zero).  All ranks make the same exchanges in the same order. */
#define RIB_TP_MAX_RANKS 8
#define RIB_EPI_PEER_PARTIAL 3 /* FP32 W x -> slot `rank` of every rank's buffer */

typedef struct rib_tp_exchange {
  int world, rank;
  uint64_t buf[RIB_TP_MAX_RANKS]; /* per rank: its exchange buffer (peer mapping) */
  uint64_t epoch;                  /* device address, u64                         */
  uint64_t done;                   /* device address, u32                         */
  int slot;                        /* words per rank slot (>= every N exchanged)  */
} rib_tp_exchange;

size_t rib_tp_buffer_bytes(int world, int slot);

/* rib_gemv with the exchange (ex may be NULL when neither is used):
 *   in_sum   x is the residual stream; the input is
 *            bf16(x + bf16(sum of the last exchange's partials)), K <= slot,
 *            and x_out [K] receives it (the next residual).
 *   epi      RIB_EPI_NONE, RIB_EPI_SWIGLU or RIB_EPI_PEER_PARTIAL (N <= slot;
 *            y unused).  out_f32 with RIB_EPI_NONE only. */
int rib_gemv_tp(const void *W, int N, int K, const void *x, const void *nw,
                int epi, int out_f32, void *y, const rib_tp_exchange *ex,
                int in_sum, void *x_out, void *stream);

/* Greedy token over the ranks' logit slices: x [n] FP32 holds logits
 * [index_offset, index_offset + n) of the vocabulary; every rank gets the
 * global argmax (the first index on ties) in out[0].  One exchange. */
int rib_argmax_f32_tp(const float *x, int n, int index_offset, int32_t *out,
                      void *workspace, const rib_tp_exchange *ex,
                      void *stream);

/* ------------------------------------------------------------------------ *
 * Tensor parallelism of the prefill projections: the exchange after the
 * row-parallel O and down GEMMs of Engine.prefill
 * (agent-test/v2/engine.py:111-116, the add_rms after each projection,
 * agent-test/v2/kernels.py:227-268), fused over NVLink peer memory in place
 * of an NCCL all-reduce.  Rows [o rpo, (o + 1) rpo) belong to rank o,
 * rpo = ceil(M / world).
 *
 *   rib_gemm_tp_partial    FP32 A W^T, each row stored straight into its
 *                          owner rank's receive slot for this rank (a
 *                          reduce-scatter inside the tcgen05 GEMM).
 *   rib_tp_reduce_add_rms  every rank's owned rows summed in rank order,
 *                          rounded to BF16 and stored into every rank's
 *                          gather buffer; then on every rank, for all M
 *                          rows, residual = bf16(residual + r) and, when
 *                          norm_w is given, out = the RMSNorm of it (the
 *                          rounding of rib_add_rms).
 *
 * Call them in pairs, with the same M, on every rank in the same order.
 * Exchange buffer of one rank: rib_tp_prefill_buffer_bytes(world,
 * rows_cap, hidden) bytes, zeroed, shared through rib_peer_buffer_alloc /
 * _open.  epoch: the pair's number, larger than every epoch used before on
 * these buffers and the same on every rank.  Waits for other ranks are
 * bounded (rib_set_wait_limit_ns); after one runs out
 * (rib_take_device_status() == RIB_ETIMEOUT) the buffers must be freed and
 * new ones made. */
typedef struct rib_tp_prefill_exchange {
  int world, rank;
  uint64_t buf[RIB_TP_MAX_RANKS]; /* per rank: its exchange buffer (peer mapping) */
  int rows_cap;                    /* rows the buffers hold (M <= rows_cap)        */
  int hidden;                      /* N of the projections: 256, 512, 1024, 2048   */
} rib_tp_prefill_exchange;

size_t rib_tp_prefill_buffer_bytes(int world, int rows_cap, int hidden);

/* A [M][K] BF16 (K % 64 == 0), W [hidden][K] BF16 (this rank's columns). */
int rib_gemm_tp_partial(const void *A, int M, int K, const void *W,
                        const rib_tp_prefill_exchange *ex, void *stream);

/* residual [M][hidden] BF16 in/out; norm_w [hidden] BF16 or NULL; out
 * [M][hidden] BF16 (unused when norm_w is NULL). */
int rib_tp_reduce_add_rms(const rib_tp_prefill_exchange *ex, int M,
                          unsigned long long epoch, void *residual,
                          const void *norm_w, void *out, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* RIB_ATTENTION_H */
