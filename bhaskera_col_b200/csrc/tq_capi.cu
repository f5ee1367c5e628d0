// tq_capi.cu — extern "C" boundary: argument validation, error reporting and
// dispatch to the kernels.  See include/tq_b200.h for the contract.
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <nvtx3/nvToolsExt.h>

#include "tq_common.cuh"
#include "tq_internal.h"

namespace tq {

// An NVTX range over one entry point (host side: the span in which it
// validates and enqueues its kernels), so a profiler's timeline shows the
// append, decode, decode-step (with the fused gather) and prefill calls.
// NVTX does nothing unless a profiler is attached.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int launch_result(cudaError_t e, const char* what) {
  if (e == cudaSuccess) e = cudaGetLastError();
  else cudaGetLastError();   // clear the sticky launch error
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

// Kernel attributes and device properties are queried once per (device,
// kernel) and cached, so that launches made while a stream is being captured
// into a CUDA graph issue nothing but the kernels themselves.
static std::mutex g_attr_mu;
static std::map<std::pair<int, const void*>, size_t> g_smem_set;
static std::map<std::tuple<int, const void*, size_t, int>, int> g_occ;
static std::map<int, int> g_sms;

static int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int set_smem_attr(const void* kernel, size_t bytes) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto key = std::make_pair(dev, kernel);
  auto it = g_smem_set.find(key);
  if (it != g_smem_set.end() && it->second >= bytes) return TQ_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)bytes);
  if (e != cudaSuccess) {
    set_error("cudaFuncSetAttribute(%zu bytes of shared memory): %s", bytes, cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  g_smem_set[key] = bytes;
  return TQ_OK;
}

int occupancy(const void* kernel, int threads, size_t smem) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto key = std::make_tuple(dev, kernel, smem, threads);
  auto it = g_occ.find(key);
  if (it != g_occ.end()) return it->second;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem) != cudaSuccess)
    occ = 1;
  g_occ[key] = occ;
  return occ;
}

int device_sm_count() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(g_attr_mu);
  auto it = g_sms.find(dev);
  if (it != g_sms.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 148;
  g_sms[dev] = n;
  return n;
}

static bool valid_dtype(int d) { return d == TQ_F32 || d == TQ_F16 || d == TQ_BF16; }

static int check_geom(const tq_geom* g, const char* fn) {
  if (!g) { set_error("%s: geometry is NULL", fn); return TQ_ERR_INVALID; }
  if (g->head_dim < 32 || g->head_dim > 256 || g->head_dim % 32) {
    set_error("%s: head_dim must be a multiple of 32 in [32, 256], got %d", fn, g->head_dim);
    return TQ_ERR_INVALID;
  }
  if (g->key_bits < 1 || g->key_bits > 8 || g->value_bits < 1 || g->value_bits > 8) {
    set_error("%s: bit widths must be in [1, 8], got key_bits=%d value_bits=%d", fn,
              g->key_bits, g->value_bits);
    return TQ_ERR_INVALID;
  }
  return TQ_OK;
}

static int check_tables(const tq_geom* g, const tq_tables* t, const char* fn) {
  if (!t || !t->k_centroids || !t->k_boundaries || !t->v_centroids || !t->v_boundaries || !t->rot ||
      !t->rot_t) {
    set_error("%s: a codebook or rotation table pointer is NULL", fn);
    return TQ_ERR_INVALID;
  }
  if (g->qjl && (!t->qjl || !t->qjl_t)) {
    set_error("%s: qjl enabled but the QJL matrix is NULL", fn);
    return TQ_ERR_INVALID;
  }
  const uintptr_t a = reinterpret_cast<uintptr_t>(t->rot_t) | reinterpret_cast<uintptr_t>(t->qjl_t);
  if (a % 16) { set_error("%s: transposed tables must be 16-byte aligned", fn); return TQ_ERR_INVALID; }
  return TQ_OK;
}

static int check_cache(const tq_cache* c, const char* fn) {
  if (!c || !c->pages || c->streams <= 0 || c->pages_per_stream <= 0) {
    set_error("%s: invalid cache descriptor", fn);
    return TQ_ERR_INVALID;
  }
  if (reinterpret_cast<uintptr_t>(c->pages) % 16) {
    set_error("%s: page storage must be 16-byte aligned", fn);
    return TQ_ERR_INVALID;
  }
  if (c->block_table &&
      (c->block_table_stride < c->pages_per_stream || c->num_blocks <= 0 ||
       reinterpret_cast<uintptr_t>(c->block_table) % 4)) {
    set_error("%s: block table needs stride >= pages_per_stream (%lld), num_blocks > 0 and "
              "4-byte alignment", fn, (long long)c->pages_per_stream);
    return TQ_ERR_INVALID;
  }
  return TQ_OK;
}

static int check_t4(const tq_tensor4* x, const char* what, const char* fn) {
  if (!x || !x->data) { set_error("%s: %s is NULL", fn, what); return TQ_ERR_INVALID; }
  if (!valid_dtype(x->dtype)) { set_error("%s: %s has unsupported dtype %d", fn, what, x->dtype); return TQ_ERR_INVALID; }
  for (int i = 0; i < 4; ++i)
    if (x->shape[i] < 0) { set_error("%s: %s has a negative extent", fn, what); return TQ_ERR_INVALID; }
  return TQ_OK;
}

}  // namespace tq

using namespace tq;

extern "C" {

const char* tq_last_error(void) { return g_err; }

int32_t tq_version(void) { return 1; }

int64_t tq_page_bytes(const tq_geom* g) {
  if (check_geom(g, "tq_page_bytes") != TQ_OK) return -1;
  return make_geom(g->head_dim, g->key_bits, g->value_bits, g->qjl).page_bytes;
}

int32_t tq_quantize_rotated(const float* y, int64_t n, const float* boundaries,
                            int32_t n_boundaries, int16_t* codes, void* stream) {
  if (n < 0 || (n > 0 && (!y || !codes || !boundaries)) || n_boundaries < 1 || n_boundaries > 255) {
    set_error("tq_quantize_rotated: invalid arguments (n=%lld, n_boundaries=%d)", (long long)n,
              n_boundaries);
    return TQ_ERR_INVALID;
  }
  return launch_quantize_rotated(y, n, boundaries, n_boundaries, codes, (cudaStream_t)stream);
}

int32_t tq_append(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                  const tq_tensor4* k, const tq_tensor4* v, int64_t pos, void* stream) {
  NvtxRange range("tq_append");
  const char* fn = "tq_append";
  int rc;
  if ((rc = check_geom(g, fn)) || (rc = check_tables(g, t, fn)) || (rc = check_cache(c, fn)) ||
      (rc = check_t4(k, "k", fn)) || (rc = check_t4(v, "v", fn)))
    return rc;
  if (g->head_dim > 128) {
    set_error("%s: head_dim %d > 128 is not supported by the append kernel", fn, g->head_dim);
    return TQ_ERR_INVALID;
  }
  for (int i = 0; i < 4; ++i)
    if (k->shape[i] != v->shape[i]) { set_error("%s: k and v shapes differ", fn); return TQ_ERR_INVALID; }
  if (k->shape[3] != g->head_dim) {
    set_error("%s: last dim %lld != head_dim %d", fn, (long long)k->shape[3], g->head_dim);
    return TQ_ERR_INVALID;
  }
  if (k->shape[0] * k->shape[1] != c->streams) {
    set_error("%s: B*H = %lld does not match the cache's %lld streams", fn,
              (long long)(k->shape[0] * k->shape[1]), (long long)c->streams);
    return TQ_ERR_INVALID;
  }
  if (pos < 0 || pos + k->shape[2] > c->pages_per_stream * TQ_PAGE_TOKENS) {
    set_error("%s: tokens [%lld, %lld) exceed the capacity of %lld tokens", fn, (long long)pos,
              (long long)(pos + k->shape[2]), (long long)(c->pages_per_stream * TQ_PAGE_TOKENS));
    return TQ_ERR_INVALID;
  }
  return launch_append(g, t, c, k, v, pos, (cudaStream_t)stream);
}

int32_t tq_dequantize(const tq_geom* g, const tq_tables* t, const tq_cache* c, int64_t t0,
                      int64_t t1, const tq_tensor4* k_out, const tq_tensor4* v_out, void* stream) {
  NvtxRange range("tq_dequantize");
  const char* fn = "tq_dequantize";
  int rc;
  if ((rc = check_geom(g, fn)) || (rc = check_tables(g, t, fn)) || (rc = check_cache(c, fn)))
    return rc;
  if (k_out && (rc = check_t4(k_out, "k_out", fn))) return rc;
  if (v_out && (rc = check_t4(v_out, "v_out", fn))) return rc;
  if (t0 < 0 || t1 < t0 || t1 > c->pages_per_stream * TQ_PAGE_TOKENS) {
    set_error("%s: token range [%lld, %lld) out of bounds", fn, (long long)t0, (long long)t1);
    return TQ_ERR_INVALID;
  }
  const tq_tensor4* o[2] = {k_out, v_out};
  for (int w = 0; w < 2; ++w) {
    if (!o[w]) continue;
    if (o[w]->shape[0] * o[w]->shape[1] != c->streams || o[w]->shape[2] != t1 - t0 ||
        o[w]->shape[3] != g->head_dim) {
      set_error("%s: output view shape does not match (streams, t1-t0, head_dim)", fn);
      return TQ_ERR_INVALID;
    }
  }
  return launch_dequant(g, t, c, t0, t1, k_out, v_out, (cudaStream_t)stream);
}

static int check_decode(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                        const tq_decode_args* a, const char* fn) {
  int rc;
  if ((rc = check_geom(g, fn)) || (rc = check_tables(g, t, fn)) || (rc = check_cache(c, fn)))
    return rc;
  if (!a) { set_error("%s: args is NULL", fn); return TQ_ERR_INVALID; }
  if ((rc = check_t4(a->q, "q", fn)) || (rc = check_t4(a->out, "out", fn))) return rc;
  const int64_t B = a->q->shape[0];
  if (B <= 0 || c->streams % B) { set_error("%s: batch does not divide the stream count", fn); return TQ_ERR_INVALID; }
  const int64_t Hkv = c->streams / B;
  if (a->num_q_heads <= 0 || a->num_q_heads % Hkv || a->q->shape[1] != a->num_q_heads ||
      a->q->shape[2] != 1 || a->q->shape[3] != g->head_dim) {
    set_error("%s: q must be (B, Hq, 1, D) with Hq a multiple of Hkv=%lld", fn, (long long)Hkv);
    return TQ_ERR_INVALID;
  }
  for (int i = 0; i < 4; ++i)
    if (a->out->shape[i] != a->q->shape[i]) { set_error("%s: out shape != q shape", fn); return TQ_ERR_INVALID; }
  if (a->n_tokens < 0 || a->n_tokens > c->pages_per_stream * TQ_PAGE_TOKENS) {
    set_error("%s: n_tokens=%lld exceeds the cache capacity", fn, (long long)a->n_tokens);
    return TQ_ERR_INVALID;
  }
  if ((a->window_k == nullptr) != (a->window_v == nullptr)) {
    set_error("%s: window_k and window_v must both be given or both be NULL", fn);
    return TQ_ERR_INVALID;
  }
  if (a->seq_lens) {
    if (reinterpret_cast<uintptr_t>(a->seq_lens) % 4) {
      set_error("%s: seq_lens must be 4-byte aligned", fn);
      return TQ_ERR_INVALID;
    }
    if (a->phases != 0 && !(a->phases & TQ_PHASE_QPREP)) {
      set_error("%s: seq_lens needs the query-preparation phase (it lays out the pages)", fn);
      return TQ_ERR_INVALID;
    }
  }
  if (a->gather) {
    const tq_gather* gt = a->gather;
    if (gt->world < 1 || gt->world > TQ_MAX_PEERS || gt->rank < 0 || gt->rank >= gt->world) {
      set_error("%s: gather.world must lie in [1, %d] and rank in [0, world)", fn, TQ_MAX_PEERS);
      return TQ_ERR_INVALID;
    }
    for (int r = 0; r < gt->world; ++r)
      if (!gt->peer_out[r] || !gt->peer_flag[r] ||
          reinterpret_cast<uintptr_t>(gt->peer_flag[r]) % 8) {
        set_error("%s: gather.peer_out / peer_flag[%d] missing or misaligned", fn, r);
        return TQ_ERR_INVALID;
      }
    if (gt->peer_out[gt->rank] != a->out->data) {
      set_error("%s: gather.peer_out[rank] must be out->data", fn);
      return TQ_ERR_INVALID;
    }
    if (a->phases != 0 && !(a->phases & TQ_PHASE_MERGE)) {
      set_error("%s: a gather needs the merge phase", fn);
      return TQ_ERR_INVALID;
    }
  }
  if (a->window_k) {
    if ((rc = check_t4(a->window_k, "window_k", fn)) || (rc = check_t4(a->window_v, "window_v", fn))) return rc;
    for (int i = 0; i < 4; ++i)
      if (a->window_k->shape[i] != a->window_v->shape[i]) { set_error("%s: window shapes differ", fn); return TQ_ERR_INVALID; }
    if (a->window_k->dtype != a->window_v->dtype) { set_error("%s: window dtypes differ", fn); return TQ_ERR_INVALID; }
    if (a->window_k->shape[0] != B || a->window_k->shape[1] != Hkv || a->window_k->shape[3] != g->head_dim) {
      set_error("%s: window must be (B, Hkv, W, D)", fn);
      return TQ_ERR_INVALID;
    }
    if (a->window_k->shape[2] > 1024) { set_error("%s: window longer than 1024 tokens", fn); return TQ_ERR_INVALID; }
  }
  return TQ_OK;
}

size_t tq_decode_workspace_bytes(const tq_geom* g, const tq_cache* c, const tq_decode_args* a) {
  const char* fn = "tq_decode_workspace_bytes";
  if (check_geom(g, fn) || check_cache(c, fn) || !a || check_t4(a->q, "q", fn)) return 0;
  if (a->q->shape[0] <= 0 || c->streams % a->q->shape[0]) return 0;
  return decode_workspace_bytes(g, c, a);
}

int32_t tq_decode_attn(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                       const tq_decode_args* a, void* workspace, size_t workspace_bytes,
                       void* stream) {
  NvtxRange range("tq_decode_attn");
  const char* fn = "tq_decode_attn";
  int rc = check_decode(g, t, c, a, fn);
  if (rc) return rc;
  return launch_decode(g, t, c, a, workspace, workspace_bytes, (cudaStream_t)stream);
}

int32_t tq_decode_step(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                       const tq_tensor4* k_new, const tq_tensor4* v_new, int64_t pos,
                       const tq_decode_args* a, void* workspace, size_t workspace_bytes,
                       void* stream) {
  NvtxRange range("tq_decode_step");
  const char* fn = "tq_decode_step";
  int rc = check_decode(g, t, c, a, fn);
  if (rc) return rc;
  if ((rc = check_t4(k_new, "k_new", fn)) || (rc = check_t4(v_new, "v_new", fn))) return rc;
  if (g->head_dim > 128) {
    set_error("%s: head_dim %d > 128 is not supported by the append path", fn, g->head_dim);
    return TQ_ERR_INVALID;
  }
  for (int i = 0; i < 4; ++i)
    if (k_new->shape[i] != v_new->shape[i]) { set_error("%s: k_new and v_new shapes differ", fn); return TQ_ERR_INVALID; }
  if (k_new->shape[0] != a->q->shape[0] || k_new->shape[0] * k_new->shape[1] != c->streams ||
      k_new->shape[2] != 1 || k_new->shape[3] != g->head_dim) {
    set_error("%s: k_new/v_new must be (B, Hkv, 1, D) with B*Hkv = %lld streams", fn,
              (long long)c->streams);
    return TQ_ERR_INVALID;
  }
  if (pos < 0 || a->n_tokens != pos + 1) {
    set_error("%s: n_tokens (%lld) must equal pos + 1 (%lld)", fn, (long long)a->n_tokens,
              (long long)(pos + 1));
    return TQ_ERR_INVALID;
  }
  StepInput step{k_new, v_new, pos};
  return launch_decode(g, t, c, a, workspace, workspace_bytes, (cudaStream_t)stream, &step);
}

int32_t tq_prefill_attn(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                        const tq_prefill_args* a, void* stream) {
  NvtxRange range("tq_prefill_attn");
  const char* fn = "tq_prefill_attn";
  int rc;
  if ((rc = check_geom(g, fn)) || (rc = check_tables(g, t, fn)) || (rc = check_cache(c, fn)))
    return rc;
  if (!a) { set_error("%s: args are NULL", fn); return TQ_ERR_INVALID; }
  if ((rc = check_t4(a->q, "q", fn)) || (rc = check_t4(a->out, "out", fn))) return rc;
  if (!t->rot_f16 || reinterpret_cast<uintptr_t>(t->rot_f16) % 16) {
    set_error("%s: tables.rot_f16 (R as fp16, 16-byte aligned) is required", fn);
    return TQ_ERR_INVALID;
  }
  if (a->engine < 0 || a->engine > 3) {
    set_error("%s: engine must be 0 (fastest), 1 (mma.sync), 2 or 3 (tcgen05, 128 or 256 "
              "rows per CTA), got %d", fn, a->engine);
    return TQ_ERR_INVALID;
  }
  if (a->engine >= 2 && !prefill_tc_applies(g)) {
    set_error("%s: no tcgen05 kernel for head_dim %d, key_bits %d, value_bits %d", fn,
              g->head_dim, g->key_bits, g->value_bits);
    return TQ_ERR_INVALID;
  }
  if (!prefill_supported(g->head_dim, g->key_bits, g->value_bits) &&
      !(a->engine != 1 && prefill_tc_applies(g))) {
    set_error("%s: no kernel for head_dim %d, key_bits %d, value_bits %d (engine %d)", fn,
              g->head_dim, g->key_bits, g->value_bits, a->engine);
    return TQ_ERR_INVALID;
  }
  const tq_tensor4 *q = a->q, *o = a->out;
  for (int i = 0; i < 4; ++i)
    if (q->shape[i] != o->shape[i]) { set_error("%s: q and out shapes differ", fn); return TQ_ERR_INVALID; }
  if (q->shape[3] != g->head_dim) {
    set_error("%s: last dim %lld != head_dim %d", fn, (long long)q->shape[3], g->head_dim);
    return TQ_ERR_INVALID;
  }
  const int64_t B = q->shape[0], Hq = q->shape[1], Tq = q->shape[2];
  if (B <= 0 || c->streams % B || Hq % (c->streams / B)) {
    set_error("%s: q (B=%lld, Hq=%lld) does not match %lld streams (B * Hkv, Hq a multiple of Hkv)",
              fn, (long long)B, (long long)Hq, (long long)c->streams);
    return TQ_ERR_INVALID;
  }
  if (B * Hq > 65535) {
    set_error("%s: B * Hq = %lld exceeds the grid limit 65535", fn, (long long)(B * Hq));
    return TQ_ERR_INVALID;
  }
  int64_t W = 0;
  if (a->window_k || a->window_v) {
    if (!a->window_k || !a->window_v) {
      set_error("%s: window_k and window_v come together", fn);
      return TQ_ERR_INVALID;
    }
    if ((rc = check_t4(a->window_k, "window_k", fn)) || (rc = check_t4(a->window_v, "window_v", fn)))
      return rc;
    W = a->window_k->shape[2];
    for (int i = 0; i < 4; ++i)
      if (a->window_k->shape[i] != a->window_v->shape[i]) {
        set_error("%s: window_k and window_v shapes differ", fn);
        return TQ_ERR_INVALID;
      }
    if (a->window_k->shape[0] != B || a->window_k->shape[1] != c->streams / B ||
        a->window_k->shape[3] != g->head_dim) {
      set_error("%s: the window must be (B, Hkv, W, head_dim)", fn);
      return TQ_ERR_INVALID;
    }
    if (W > 0 && (a->engine == 1 || !prefill_tc_applies(g))) {
      set_error("%s: a residual window needs the tcgen05 kernel (head_dim 128, 2-4 bit codes, "
                "engine 0, 2 or 3)", fn);
      return TQ_ERR_INVALID;
    }
    if (W > 0 && (!a->workspace || a->workspace_bytes < tq_prefill_workspace_bytes(g, c, a) ||
                  reinterpret_cast<uintptr_t>(a->workspace) % 256)) {
      set_error("%s: a residual window needs a 256-byte aligned workspace of %zu bytes", fn,
                tq_prefill_workspace_bytes(g, c, a));
      return TQ_ERR_WORKSPACE;
    }
  }
  if (a->n_tokens < Tq || a->n_tokens < W ||
      a->n_tokens - W > c->pages_per_stream * TQ_PAGE_TOKENS) {
    set_error("%s: n_tokens %lld must lie in [Tq = %lld, capacity %lld + window %lld]", fn,
              (long long)a->n_tokens, (long long)Tq,
              (long long)(c->pages_per_stream * TQ_PAGE_TOKENS), (long long)W);
    return TQ_ERR_INVALID;
  }
  if (!(a->scale > 0.f)) { set_error("%s: scale must be positive", fn); return TQ_ERR_INVALID; }
  uint32_t* status = device_status_word();
  if (!status) { set_error("%s: device status word unavailable", fn); return TQ_ERR_CUDA; }
  return launch_prefill(g, t, c, a, status, (cudaStream_t)stream);
}

size_t tq_prefill_workspace_bytes(const tq_geom* g, const tq_cache* c, const tq_prefill_args* a) {
  if (!g || !c || !a || !a->window_k || a->window_k->shape[2] <= 0) return 0;
  // the window rotated into fp16, K then V: [streams][W][head_dim] each
  const size_t one = (size_t)c->streams * (size_t)a->window_k->shape[2] * (size_t)g->head_dim * 2;
  return 2 * ((one + 255) & ~(size_t)255);
}

int32_t tq_workspace_status(void* workspace, uint32_t* status, void* stream) {
  if (!workspace || !status) { set_error("tq_workspace_status: NULL argument"); return TQ_ERR_INVALID; }
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(status, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) {
    set_error("tq_workspace_status: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return *status ? TQ_ERR_DEVICE : TQ_OK;
}

int32_t tq_append_tensor_core(const tq_geom* g, const tq_tables* t, const tq_tensor4* k,
                              const tq_tensor4* v) {
  if (!g || !t || !k || !v) return 0;
  return append_tc_applies(g, t, k, v) ? 1 : 0;
}

int32_t tq_prefill_tensor_core(const tq_geom* g) {
  if (!g || check_geom(g, "tq_prefill_tensor_core")) return 0;
  return prefill_tc_applies(g) ? 1 : 0;
}

int32_t tq_device_status(uint32_t* status, void* stream) {
  if (!status) { set_error("tq_device_status: NULL argument"); return TQ_ERR_INVALID; }
  return read_tc_status(status, (cudaStream_t)stream);
}

int32_t tq_shared_alloc(size_t bytes, void** dptr, void* handle) {
  if (!dptr || !handle || bytes == 0) { set_error("tq_shared_alloc: bad argument"); return TQ_ERR_INVALID; }
  static_assert(sizeof(cudaIpcMemHandle_t) <= TQ_SHARED_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_error("tq_shared_alloc: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  memset(handle, 0, TQ_SHARED_HANDLE_BYTES);
  memcpy(handle, &h, sizeof(h));
  *dptr = p;
  return TQ_OK;
}

int32_t tq_shared_open(const void* handle, void** dptr) {
  if (!dptr || !handle) { set_error("tq_shared_open: bad argument"); return TQ_ERR_INVALID; }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) { set_error("tq_shared_open: %s", cudaGetErrorString(e)); return TQ_ERR_CUDA; }
  return TQ_OK;
}

int32_t tq_shared_close(void* dptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dptr);
  if (e != cudaSuccess) { set_error("tq_shared_close: %s", cudaGetErrorString(e)); return TQ_ERR_CUDA; }
  return TQ_OK;
}

int32_t tq_shared_free(void* dptr) {
  cudaError_t e = cudaFree(dptr);
  if (e != cudaSuccess) { set_error("tq_shared_free: %s", cudaGetErrorString(e)); return TQ_ERR_CUDA; }
  return TQ_OK;
}

// ---------------------------------------------------------------------------
// tables from host arrays
// ---------------------------------------------------------------------------
namespace {

struct TableLayout {
  size_t kc, kb, vc, vb, rot, rot_t, qjl, qjl_t, bf3, f16, qb, total;
};

TableLayout table_layout(const tq_geom* g) {
  const size_t D = (size_t)g->head_dim, DD = D * D;
  TableLayout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = (off + bytes + 255) & ~(size_t)255;
    return at;
  };
  L.kc = take(((size_t)1 << g->key_bits) * 4);
  L.kb = take((((size_t)1 << g->key_bits) - 1) * 4 + 4);
  L.vc = take(((size_t)1 << g->value_bits) * 4);
  L.vb = take((((size_t)1 << g->value_bits) - 1) * 4 + 4);
  L.rot = take(DD * 4);
  L.rot_t = take(DD * 4);
  L.qjl = g->qjl ? take(DD * 4) : 0;
  L.qjl_t = g->qjl ? take(DD * 4) : 0;
  L.bf3 = D == 128 ? take(6 * DD * 2) : 0;
  L.f16 = take(DD * 2);
  L.qb = g->qjl && D == 128 ? take(DD * 2) : 0;
  L.total = off;
  return L;
}

uint16_t bf16_bits(float x) {
  const __nv_bfloat16 h = __float2bfloat16_rn(x);
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}

float bf16_value(uint16_t u) {
  const uint32_t w = (uint32_t)u << 16;
  float f;
  memcpy(&f, &w, 4);
  return f;
}

}  // namespace

size_t tq_tables_bytes(const tq_geom* g) {
  if (check_geom(g, "tq_tables_bytes")) return 0;
  return table_layout(g).total;
}

int32_t tq_init_tables(const tq_geom* g, const float* k_centroids, const float* k_boundaries,
                       const float* v_centroids, const float* v_boundaries, const float* rot,
                       const float* qjl, void* device_buf, size_t device_bytes, tq_tables* t,
                       void* stream) {
  const char* fn = "tq_init_tables";
  if (int rc = check_geom(g, fn)) return rc;
  if (!k_centroids || !k_boundaries || !v_centroids || !v_boundaries || !rot || !t ||
      !device_buf || (g->qjl && !qjl)) {
    set_error("%s: a table, the output or the device buffer is NULL", fn);
    return TQ_ERR_INVALID;
  }
  const TableLayout L = table_layout(g);
  if (device_bytes < L.total || reinterpret_cast<uintptr_t>(device_buf) % 256) {
    set_error("%s: device buffer of %zu bytes (256-byte aligned) needed, %zu given", fn, L.total,
              device_bytes);
    return TQ_ERR_INVALID;
  }
  const int D = g->head_dim;
  const size_t DD = (size_t)D * D;
  std::vector<uint8_t> host(L.total, 0);
  auto put = [&](size_t off, const void* src, size_t bytes) { memcpy(host.data() + off, src, bytes); };
  put(L.kc, k_centroids, ((size_t)1 << g->key_bits) * 4);
  put(L.kb, k_boundaries, (((size_t)1 << g->key_bits) - 1) * 4);
  put(L.vc, v_centroids, ((size_t)1 << g->value_bits) * 4);
  put(L.vb, v_boundaries, (((size_t)1 << g->value_bits) - 1) * 4);
  put(L.rot, rot, DD * 4);
  float* rt = reinterpret_cast<float*>(host.data() + L.rot_t);
  uint16_t* f16 = reinterpret_cast<uint16_t*>(host.data() + L.f16);
  for (int i = 0; i < D; ++i)
    for (int j = 0; j < D; ++j) {
      rt[(size_t)j * D + i] = rot[(size_t)i * D + j];
      const __half h = __float2half_rn(rot[(size_t)i * D + j]);
      memcpy(&f16[(size_t)i * D + j], &h, 2);
    }
  if (g->qjl) {
    put(L.qjl, qjl, DD * 4);
    float* st = reinterpret_cast<float*>(host.data() + L.qjl_t);
    for (int i = 0; i < D; ++i)
      for (int j = 0; j < D; ++j) st[(size_t)j * D + i] = qjl[(size_t)i * D + j];
  }
  if (D == 128) {
    // R = hi + mid + lo in bf16, each rounded to nearest from the fp32
    // remainder; rows in K quad order ([0]) and V octet order ([1])
    uint16_t* b3 = reinterpret_cast<uint16_t*>(host.data() + L.bf3);
    for (int o = 0; o < 2; ++o)
      for (int p = 0; p < D; ++p) {
        const int row = o == 0 ? k_coord_at(p, D) : v_coord_at(p, D);
        for (int c = 0; c < D; ++c) {
          const float x = rot[(size_t)row * D + c];
          const uint16_t hi = bf16_bits(x);
          const float r1 = x - bf16_value(hi);
          const uint16_t mid = bf16_bits(r1);
          const uint16_t lo = bf16_bits(r1 - bf16_value(mid));
          const size_t at = (((size_t)o * 3) * D + p) * D + c;
          b3[at] = hi;
          b3[at + DD] = mid;
          b3[at + 2 * DD] = lo;
        }
      }
  }
  // S in bf16 for the tensor-core sketch, rows and columns in K quad order,
  // only when every entry is exactly a bf16 value
  bool qb_ok = g->qjl && D == 128;
  if (qb_ok) {
    for (size_t i = 0; i < DD && qb_ok; ++i) qb_ok = bf16_value(bf16_bits(qjl[i])) == qjl[i];
    uint16_t* qb = reinterpret_cast<uint16_t*>(host.data() + L.qb);
    for (int p = 0; qb_ok && p < D; ++p)
      for (int c = 0; c < D; ++c)
        qb[(size_t)p * D + c] = bf16_bits(qjl[(size_t)k_coord_at(p, D) * D + k_coord_at(c, D)]);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(device_buf, host.data(), L.total, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_error("%s: %s", fn, cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  uint8_t* base = static_cast<uint8_t*>(device_buf);
  t->k_centroids = reinterpret_cast<const float*>(base + L.kc);
  t->k_boundaries = reinterpret_cast<const float*>(base + L.kb);
  t->v_centroids = reinterpret_cast<const float*>(base + L.vc);
  t->v_boundaries = reinterpret_cast<const float*>(base + L.vb);
  t->rot = reinterpret_cast<const float*>(base + L.rot);
  t->rot_t = reinterpret_cast<const float*>(base + L.rot_t);
  t->qjl = g->qjl ? reinterpret_cast<const float*>(base + L.qjl) : nullptr;
  t->qjl_t = g->qjl ? reinterpret_cast<const float*>(base + L.qjl_t) : nullptr;
  t->rot_bf16x3 = D == 128 ? reinterpret_cast<const uint16_t*>(base + L.bf3) : nullptr;
  t->rot_f16 = reinterpret_cast<const uint16_t*>(base + L.f16);
  t->qjl_bf16 = qb_ok ? reinterpret_cast<const uint16_t*>(base + L.qb) : nullptr;
  return TQ_OK;
}

}  // extern "C"
