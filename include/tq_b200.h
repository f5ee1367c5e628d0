/*
 * tq_b200.h — C ABI of the B200 (sm_100a) TurboQuant KV-cache kernels.
 *
 * Every entry point takes raw device pointers, explicit sizes and strides,
 * and a cudaStream_t passed as `void*`.  Nothing here allocates device
 * memory: scratch ("workspace") is supplied by the caller and sized with the
 * matching *_workspace_bytes() query.  Work is stream-ordered and no entry
 * point synchronises the host, except the init-time tq_init_tables and the
 * status reads.  Every function returns TQ_OK (0) or a
 * negative status; tq_last_error() gives a thread-local message for the last
 * failure on the calling thread.
 *
 * Reference interfaces replaced (aditya25058/Bhaskera_col, paths relative to
 * the project root):
 *   tq_quantize_rotated  FastLloydMaxCodebook.quantize
 *                        src/bhaskera/inference/kv_cache.py:105-113
 *   tq_append            _LayerKVStore._compress_chunk (norm, rotate,
 *                        bucketize, store)  kv_cache.py:355-420
 *   tq_dequantize        _LayerKVStore._decode_range  kv_cache.py:422-439
 *   tq_decode_attn       the HF attention over TurboQuantKVCache.update()'s
 *                        output (torch SDPA, GQA), reached from
 *                        src/bhaskera/inference/engine.py:389 through
 *                        kv_cache.py:580-589
 *   tq_prefill_attn      same, causal multi-token case
 *
 * Packed layout (per layer): an array of streams (stream = b * Hkv + h, the
 * reference's B*H flattening at kv_cache.py:364-365), each an array of
 * pages of TQ_PAGE_TOKENS tokens.  A page holds, in order:
 *   kcodes [64][D*kb/8]   K codes, quad order, LSB-first bit stream
 *   vcodes [64][D*vb/8]   V codes, octet order, LSB-first bit stream
 *   kqjl   [64][D/8]      QJL residual signs (only when qjl != 0)
 *   knorm  [64] fp16      ||k||
 *   vnorm  [64] fp16      ||v||
 *   krnorm [64] fp16      ||k|| * ||y - c[idx]||  (only when qjl != 0)
 * Quad order: quad t (t = 0..3) lists, for each 16-coordinate chunk j,
 * coordinates 16j+2t, 16j+2t+1, 16j+2t+8, 16j+2t+9.  Octet order: octet g
 * (g = 0..7) lists coordinates g, g+8, g+16, ...
 */
#ifndef TQ_B200_H
#define TQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TQ_PAGE_TOKENS 64

/* status codes */
#define TQ_OK 0
#define TQ_ERR_INVALID (-1)     /* bad argument / unsupported shape        */
#define TQ_ERR_CUDA (-2)        /* a CUDA runtime call or launch failed    */
#define TQ_ERR_WORKSPACE (-3)   /* workspace missing or too small          */
#define TQ_ERR_DEVICE (-4)      /* a kernel reported a device-side error   */

/* element types */
#define TQ_F32 0
#define TQ_F16 1
#define TQ_BF16 2

/* device status word bits (written by kernels into the workspace) */
#define TQ_DEV_WAIT_TIMEOUT 1u  /* a bounded mbarrier wait ran out          */
#define TQ_DEV_BAD_BLOCK 2u     /* a block-table entry was outside the pool */

typedef struct tq_geom {
  int32_t head_dim;    /* D: multiple of 32, 32..256                        */
  int32_t key_bits;    /* 1..8                                               */
  int32_t value_bits;  /* 1..8                                               */
  int32_t qjl;         /* 1: store the 1-bit QJL residual sketch of K        */
} tq_geom;

/* Per-layer constant tables, all fp32 device pointers. */
typedef struct tq_tables {
  const float* k_centroids;   /* [2^kb]                                     */
  const float* k_boundaries;  /* [2^kb - 1], ascending                       */
  const float* v_centroids;   /* [2^vb]                                      */
  const float* v_boundaries;  /* [2^vb - 1]                                  */
  const float* rot;           /* R [D][D] row-major; y = x R^T               */
  const float* qjl;           /* S [D][D] row-major (NULL when qjl == 0)     */
  const float* rot_t;         /* R^T [D][D] row-major                        */
  const float* qjl_t;         /* S^T [D][D] row-major (NULL when qjl == 0)   */
  /* Optional, head_dim 128 only: R as three bf16 terms (hi = bf16(R),
   * mid = bf16(R - hi), lo = bf16(R - hi - mid)) with rows in packed order,
   * [2][3][D][D] bf16: [0][s][p] = term s of R row k_order[p] (K quad order),
   * [1][s][p] = term s of R row v_order[p] (V octet order).  When set,
   * tq_append runs the rotation of bf16 inputs on the tensor cores; NULL
   * keeps every append on the CUDA-core kernel. */
  const uint16_t* rot_bf16x3;
  /* R [D][D] fp16, row-major: required by tq_prefill_attn, unused elsewhere. */
  const uint16_t* rot_f16;
  /* Optional, head_dim 128 with qjl only: S in bf16, [D][D], rows and columns
   * in K quad order ([p][c] = S[k_order[p]][k_order[c]]).  Set only when every
   * entry of S is exactly a bf16 value (the library's own S is); then
   * tq_append computes the QJL sketch of bf16 inputs on the tensor cores with
   * the same signs as the CUDA-core kernel up to fp32 rounding of z. */
  const uint16_t* qjl_bf16;
} tq_tables;

/* Packed cache of one layer. */
typedef struct tq_cache {
  uint8_t* pages;             /* [streams][pages_per_stream][page_bytes], or
                                 with a block table a pool of num_blocks pages */
  int64_t streams;            /* B * Hkv                                     */
  int64_t pages_per_stream;   /* capacity in pages (logical, per stream)     */
  /* Optional paged layout (vLLM-style block tables): logical page p of stream
   * s lives at pool page block_table[s * block_table_stride + p].  NULL: the
   * contiguous layout above.  Entries outside [0, num_blocks) are never
   * dereferenced: reads take pool page 0, writes are dropped, and
   * TQ_DEV_BAD_BLOCK is set in the status word. */
  const int32_t* block_table;
  int64_t block_table_stride; /* >= pages_per_stream                          */
  int64_t num_blocks;         /* pages in the pool                            */
} tq_cache;

/* A strided 4-d tensor view (B, H, T, D); strides in elements. */
typedef struct tq_tensor4 {
  void* data;
  int32_t dtype;              /* TQ_F32 / TQ_F16 / TQ_BF16                   */
  int64_t shape[4];
  int64_t stride[4];
} tq_tensor4;

const char* tq_last_error(void);
int32_t tq_version(void);
int64_t tq_page_bytes(const tq_geom* g);

/* One layer's tables from host arrays, for callers without PyTorch.
 * tq_tables_bytes(g): device bytes the tables need (0 on a bad geometry).
 * tq_init_tables copies the codebooks (fp32: centroids [2^bits], boundaries
 * [2^bits - 1]), R and, with g->qjl, S ([D][D] row-major fp32) into
 * `device_buf` (>= tq_tables_bytes(g) bytes, 256-byte aligned), derives R^T,
 * S^T, R in fp16 and, for head_dim 128, the three bf16 terms of R in packed
 * row order, and points *t into the buffer.  It synchronises `stream` once
 * (an init-time call; the host arrays may be freed on return).  Replaces the
 * table set-up of _LayerKVStore.__init__ (kv_cache.py:270-311): R from
 * _generate_rotation_matrix, codebooks from FastLloydMaxCodebook.get. */
size_t tq_tables_bytes(const tq_geom* g);
int32_t tq_init_tables(const tq_geom* g, const float* k_centroids, const float* k_boundaries,
                       const float* v_centroids, const float* v_boundaries, const float* rot,
                       const float* qjl, void* device_buf, size_t device_bytes, tq_tables* t,
                       void* stream);

/* Bit-exact scalar quantiser: codes[i] = #{ j : boundaries[j] < y[i] }
 * (torch.bucketize, right=False) for n fp32 values, int16 output.
 * Replaces FastLloydMaxCodebook.quantize (kv_cache.py:105-113). */
int32_t tq_quantize_rotated(const float* y, int64_t n, const float* boundaries,
                            int32_t n_boundaries, int16_t* codes,
                            void* stream);

/* Fused append of tokens [pos, pos + T) of every stream: fp32 norm,
 * u = x / max(n, 1e-8), y = u R^T, codes = bucketize(y), pack, fp16 norms,
 * optional QJL sign sketch of the rotated residual.  k and v are (B, Hkv,
 * T, D) views with B * Hkv == cache->streams.
 * Replaces _LayerKVStore._compress_chunk (kv_cache.py:355-420). */
int32_t tq_append(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                  const tq_tensor4* k, const tq_tensor4* v, int64_t pos,
                  void* stream);

/* Dequantise tokens [t0, t1) of every stream into dense K/V views
 * (B, Hkv, t1 - t0, D): x = (c[idx] R) * norm, cast to the view's dtype.
 * Either output may be NULL.  Replaces _decode_range (kv_cache.py:422-439). */
int32_t tq_dequantize(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                      int64_t t0, int64_t t1, const tq_tensor4* k_out,
                      const tq_tensor4* v_out, void* stream);

/* Single-token GQA decode attention straight off the packed cache, plus an
 * optional full-precision window of the most recent tokens (not rotated).
 * q: (B, Hq, 1, D); out: (B, Hq, 1, D); window_k/v: (B, Hkv, W, D) or NULL.
 * Keys [0, n_tokens) of every stream are attended.  scale is the softmax
 * scale (1/sqrt(D) for SDPA's default).  Workspace from
 * tq_decode_workspace_bytes(). */
/* Output all-gather fused into the decode (one process per GPU, KV heads
 * sharded over `world` ranks).  Each rank's merge kernel stores its
 * (B, Hq/world, 1, D) output block into every rank's copy of the gathered
 * buffer over peer memory (plain NVLink stores); the rank's last CTA then
 * adds 1 to every rank's arrival counter of the layer and waits (bounded,
 * TQ_DEV_WAIT_TIMEOUT in the status word on expiry) until the counter shows
 * every rank's arrival for this call, so the call completes with the
 * gathered output in place.  The arrival counter only grows; the call count
 * gives each call its target.
 * Buffers come from tq_shared_alloc / tq_shared_open.  Replaces the NCCL
 * all-gather after each layer's attention (the multi-GPU form of the
 * reference's single-process cache, kv_cache.py:516-624). */
#define TQ_MAX_PEERS 8
typedef struct tq_gather {
  int32_t world;                       /* ranks (1..TQ_MAX_PEERS)              */
  int32_t rank;                        /* this rank                            */
  void* peer_out[TQ_MAX_PEERS];        /* on rank p: this rank's output block;
                                          peer_out[rank] == out->data; the
                                          block has out's strides on every rank */
  uint32_t* peer_flag[TQ_MAX_PEERS];   /* on rank p: the layer's three words
                                          (arrivals from all ranks, rank p's
                                          finished CTAs, rank p's completed
                                          calls), zeroed once before the first
                                          call and owned by the kernels after */
} tq_gather;

typedef struct tq_decode_args {
  const tq_tensor4* q;
  const tq_tensor4* out;
  const tq_tensor4* window_k;  /* may be NULL                                */
  const tq_tensor4* window_v;  /* may be NULL                                */
  int64_t n_tokens;            /* packed tokens per stream                   */
  int64_t num_q_heads;         /* Hq (multiple of Hkv)                       */
  float scale;
  int32_t num_ctas;            /* 0: choose from the SM count                */
  int32_t phases;              /* 0: all; else OR of TQ_PHASE_* (each phase  */
                               /* reads what the previous one left in the   */
                               /* same workspace)                            */
  const tq_gather* gather;     /* NULL: out only; else the fused all-gather  */
  /* Ragged batches (continuous batching, vLLM's seq_lens): NULL, or a device
   * int32[B] whose entry b is the token count of batch row b (its streams
   * b*Hkv .. b*Hkv + Hkv - 1), clamped on the device to [0, n_tokens];
   * n_tokens is then the longest row's bound.  The decode splits only the
   * rows' real pages evenly over its CTAs.  With tq_decode_step, row b's new
   * token is stored at seq_lens[b] - 1 (nothing is stored where that is
   * negative).  Needs TQ_PHASE_QPREP in `phases` (0 = all phases). */
  const int32_t* seq_lens;
  /* Left padding (HF batched generation): NULL, or a device int32[B] whose
   * entry b is the first position row b attends; keys at earlier positions
   * (packed and window alike; window token w sits at position n_b + w, n_b
   * the row's packed tokens) take no weight.  A row whose every key is
   * masked returns zeros. */
  const int32_t* kv_start;
} tq_decode_args;

#define TQ_PHASE_QPREP 1       /* rotate + sketch the query                  */
#define TQ_PHASE_DECODE 2      /* attend the packed pages (partials)         */
#define TQ_PHASE_MERGE 4       /* combine partials + window, un-rotate       */

size_t tq_decode_workspace_bytes(const tq_geom* g, const tq_cache* c,
                                 const tq_decode_args* a);
int32_t tq_decode_attn(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                       const tq_decode_args* a, void* workspace,
                       size_t workspace_bytes, void* stream);

/* One decode step of one layer: quantise and store the new token of every
 * stream (k_new, v_new: (B, Hkv, 1, D)) at position `pos`, then attend q
 * over tokens [0, pos + 1) plus the window.  a->n_tokens must be pos + 1.
 * Same pages and outputs as tq_append(..., pos) followed by tq_decode_attn,
 * but the append is fused into the query preparation (three kernels, each
 * launched so its prologue overlaps the previous kernel).  Replaces the
 * per-layer update() + attention of a decode step (kv_cache.py:445-490 then
 * engine.py:389).  Workspace from tq_decode_workspace_bytes(). */
int32_t tq_decode_step(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                       const tq_tensor4* k_new, const tq_tensor4* v_new, int64_t pos,
                       const tq_decode_args* a, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Prefill attention straight off the packed cache: queries q (B, Hq, Tq, D)
 * at positions n_tokens - Tq .. n_tokens - 1 of every stream attend the
 * stream's tokens [0, n_tokens) (causal: a query at position p attends keys
 * <= p), GQA with Hq a multiple of Hkv; out (B, Hq, Tq, D).  Keys and values
 * are the dequantised ones, n (c[idx] R) (MSE codes; a QJL sketch is not
 * used), so the result is SDPA over what update() returns; keys
 * in a residual window (window_k/v below) enter exactly.  head_dim 64 or
 * 128; t->rot_f16 is required.  Workspace only for a window; device-side
 * wait timeouts go to the library status word (tq_device_status).  Replaces HF attention over update()'s output in a
 * prefill forward (kv_cache.py:483-488, engine.py:389). */
typedef struct tq_prefill_args {
  const tq_tensor4* q;
  const tq_tensor4* out;
  int64_t n_tokens;            /* tokens per stream, the Tq new ones included */
  float scale;                 /* softmax scale                               */
  int32_t causal;              /* 1: causal; 0: every query sees all tokens   */
  int32_t engine;              /* 0: the fastest kernel for the shape (tcgen05
                                  tensor cores where tq_prefill_tensor_core
                                  says so: 256 query rows per CTA for chunks
                                  longer than one 128-row block); 1: the
                                  mma.sync kernel; 2 / 3: the tcgen05 kernel
                                  with 128 / 256 rows per CTA                 */
  /* Left padding: NULL, or a device int32[B]: row b's keys before position
   * kv_start[b] take no weight (a query row with no key left returns zeros). */
  const int32_t* kv_start;
  /* Residual window (the reference's residual_window, kv_cache.py:461-477):
   * NULL, or (B, Hkv, W, D) dense K and V of the stream's newest W tokens,
   * which sit at positions n_tokens - W .. n_tokens - 1 after the packed
   * tokens [0, n_tokens - W).  They are attended exactly as given (rotated
   * once into fp16 in `workspace`, no quantisation).  Needs the tcgen05
   * kernel (tq_prefill_tensor_core) and a workspace of
   * tq_prefill_workspace_bytes. */
  const tq_tensor4* window_k;
  const tq_tensor4* window_v;
  void* workspace;
  size_t workspace_bytes;
} tq_prefill_args;

int32_t tq_prefill_attn(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                        const tq_prefill_args* a, void* stream);

/* Workspace bytes tq_prefill_attn needs for these arguments (the rotated
 * residual window; 0 without one). */
size_t tq_prefill_workspace_bytes(const tq_geom* g, const tq_cache* c, const tq_prefill_args* a);

/* 1 when tq_prefill_attn with engine 0 runs on the tcgen05 tensor cores for
 * this geometry (head_dim 128, key and value codes of 2 to 4 bits), else 0. */
int32_t tq_prefill_tensor_core(const tq_geom* g);

/* tq_decode_attn for callers that cannot allocate device memory (a runtime
 * that owns all device memory through its own pool, or code that must not
 * call an allocator while serving).  Same arguments and result as
 * tq_decode_attn, minus the workspace: the scratch is a fixed 8 MiB array
 * inside this library (held on every GPU that loads it until exit).  Calls
 * needing more scratch than that fail with TQ_ERR_WORKSPACE; a->phases must
 * be 0 (all phases in one call), else TQ_ERR_INVALID.  The first call on a
 * device looks the array's address up (do it before any stream capture);
 * the address is not valid after cudaDeviceReset.  Calls share the array,
 * so calls that overlap on the GPU race; serialise them.  Device-side errors
 * (TQ_DEV_WAIT_TIMEOUT, TQ_DEV_BAD_BLOCK) are recorded in the array's status
 * word, which each call clears at its start: read it with tq_noalloc_status
 * after the call and before the next one.  No counterpart in the
 * reference. */
int32_t tq_decode_attn_noalloc(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                               const tq_decode_args* a, void* stream);

/* Read and clear the status word of the current device's built-in
 * tq_decode_attn_noalloc array (blocking copy on `stream`); TQ_ERR_DEVICE
 * when a bit was set.  No counterpart in the reference. */
int32_t tq_noalloc_status(uint32_t* status, void* stream);

/* Read and clear the device status word kept at the start of a decode
 * workspace (blocking copy on `stream`). */
int32_t tq_workspace_status(void* workspace, uint32_t* status, void* stream);

/* 1 when tq_append with these arguments runs the tensor-core kernel (head_dim
 * 128, bf16 views with 16-byte aligned rows, >= 32 tokens, rot_bf16x3 set,
 * and with qjl also qjl_bf16), 0 when it runs the CUDA-core kernel.
 * Host-only query. */
int32_t tq_append_tensor_core(const tq_geom* g, const tq_tables* t, const tq_tensor4* k,
                              const tq_tensor4* v);

/* Read and clear the library's own device status word, set by kernels that
 * take no workspace (the tensor-core append: TQ_DEV_WAIT_TIMEOUT when one of
 * its bounded waits ran out).  Blocking copy on `stream`.  No reference
 * counterpart: the reference's append runs on the host. */
int32_t tq_device_status(uint32_t* status, void* stream);

/* Device memory shareable with the other processes of one node (CUDA IPC on
 * a plain allocation; no multicast object).  tq_shared_alloc returns a zeroed
 * allocation and its 64-byte handle; another process maps it with
 * tq_shared_open (peer access enabled on first use) and unmaps it with
 * tq_shared_close; the owner frees it with tq_shared_free. */
#define TQ_SHARED_HANDLE_BYTES 64
int32_t tq_shared_alloc(size_t bytes, void** dptr, void* handle);
int32_t tq_shared_open(const void* handle, void** dptr);
int32_t tq_shared_close(void* dptr);
int32_t tq_shared_free(void* dptr);

#ifdef __cplusplus
}
#endif

#endif /* TQ_B200_H */
