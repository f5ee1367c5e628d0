// tq_common.cuh — shared device helpers for the TurboQuant sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tq_b200.h"

namespace tq {

constexpr int kPageTokens = TQ_PAGE_TOKENS;

template <class T>
__host__ __device__ __forceinline__ constexpr T tmin(T a, T b) { return a < b ? a : b; }
template <class T>
__host__ __device__ __forceinline__ constexpr T tmax(T a, T b) { return a < b ? b : a; }

// ---------------------------------------------------------------------------
// Page geometry (mirrors the layout documented in tq_b200.h)
// ---------------------------------------------------------------------------
struct PageGeom {
  int D, kb, vb, qjl;
  int krow, vrow, qrow;          // bytes per token row
  int off_k, off_v, off_q;       // section offsets in bytes
  int off_kn, off_vn, off_kr;
  int page_bytes;
};

__host__ __device__ inline PageGeom make_geom(int D, int kb, int vb, int qjl) {
  PageGeom g;
  g.D = D; g.kb = kb; g.vb = vb; g.qjl = qjl;
  g.krow = D * kb / 8;
  g.vrow = D * vb / 8;
  g.qrow = qjl ? D / 8 : 0;
  int off = 0;
  g.off_k = off;  off += kPageTokens * g.krow;
  g.off_v = off;  off += kPageTokens * g.vrow;
  g.off_q = off;  off += kPageTokens * g.qrow;
  g.off_kn = off; off += 2 * kPageTokens;
  g.off_vn = off; off += 2 * kPageTokens;
  g.off_kr = off; off += qjl ? 2 * kPageTokens : 0;
  g.page_bytes = off;
  return g;
}

// Pool slot of logical page `pg` of stream `s`: contiguous (s * pps + pg) or
// through a block table.  `ok` is false for an entry outside the pool; the
// caller then reads slot 0 / drops the write and flags TQ_DEV_BAD_BLOCK.
struct PageMap {
  int64_t pps;                 // pages per stream (contiguous layout)
  const int32_t* bt;           // block table or nullptr
  int64_t bt_stride, nblocks;
};
__host__ __device__ inline PageMap page_map(const tq_cache* c) {
  PageMap m;
  m.pps = c->pages_per_stream;
  m.bt = c->block_table;
  m.bt_stride = c->block_table_stride;
  m.nblocks = c->num_blocks;
  return m;
}
__device__ __forceinline__ int64_t page_slot(const PageMap& m, int64_t s, int64_t pg, bool& ok) {
  if (m.bt == nullptr) { ok = true; return s * m.pps + pg; }
  const int64_t slot = __ldg(m.bt + s * m.bt_stride + pg);
  ok = slot >= 0 && slot < m.nblocks;
  return ok ? slot : 0;
}
// page_slot in two halves, so a loop can load the table entry of a later
// page before it waits: the raw entry, then its check.
__device__ __forceinline__ int64_t page_entry(const PageMap& m, int64_t s, int64_t pg) {
  return m.bt == nullptr ? s * m.pps + pg : (int64_t)__ldg(m.bt + s * m.bt_stride + pg);
}
__device__ __forceinline__ bool entry_ok(const PageMap& m, int64_t e) {
  return m.bt == nullptr || (e >= 0 && e < m.nblocks);
}

// Position of coordinate `coord` in the quad order of a K row.
__host__ __device__ inline int k_pos_of(int coord, int D) {
  int j = coord >> 4, r = coord & 15;
  int hi = r >> 3;                 // 0: 16j+2t(+1), 1: 16j+2t+8(+1)
  int t = (r & 7) >> 1, odd = r & 1;
  return t * (D / 4) + j * 4 + hi * 2 + odd;
}

// Position of coordinate `coord` in the octet order of a V row.
__host__ __device__ inline int v_pos_of(int coord, int D) {
  return (coord & 7) * (D / 8) + (coord >> 3);
}

// The coordinates stored at position p of a K row / a V row (inverses of
// k_pos_of and v_pos_of).
__host__ __device__ inline int k_coord_at(int p, int D) {
  const int t = p / (D / 4), e = p % (D / 4);
  const int j = e >> 2, w = e & 3;           // w: entries 16j+2t, +1, +8, +9
  return 16 * j + 2 * t + (w & 1) + 8 * (w >> 1);
}
__host__ __device__ inline int v_coord_at(int p, int D) {
  return (p / (D / 8)) + 8 * (p % (D / 8));
}

// Bit position of quad entry e (k_pos_of) inside a QJL row.
__host__ __device__ inline int qjl_bit_of(int kpos, int D) {
  int q = D / 4;
  int t = kpos / q, e = kpos % q;
  int sp = (D / 8) < 16 ? (D / 8) : 16;
  int p = e >> 1;
  int chunk = p / sp, pin = p % sp;
  return t * q + chunk * 2 * sp + ((e & 1) ? sp : 0) + pin;
}

// ---------------------------------------------------------------------------
// Element loads / stores
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_elem(const void* p, int dtype, int64_t i) {
  if (dtype == TQ_F32) return reinterpret_cast<const float*>(p)[i];
  if (dtype == TQ_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__device__ __forceinline__ void store_elem(void* p, int dtype, int64_t i, float x) {
  if (dtype == TQ_F32) reinterpret_cast<float*>(p)[i] = x;
  else if (dtype == TQ_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
}

// Number of boundaries strictly below y (torch.bucketize, right=False).
__device__ __forceinline__ int bucketize_lt(const float* b, int nb, float y) {
  int lo = 0, hi = nb;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (b[mid] < y) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---------------------------------------------------------------------------
// Warp reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (global -> shared, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// try_wait that lets the hardware suspend the thread for up to `hint_ns`
// (instead of a short system default) while the phase is incomplete, so a
// waiting warp costs no issue slots.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns) : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for a hot hand-off: polls try_wait without a suspend-time hint
// (a hinted wait resumes about 0.1 us after the phase completes) and gives up
// after about 2 s.
__device__ __forceinline__ bool mbar_wait_poll(uint64_t* bar, uint32_t parity) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      const uint64_t t = global_ns();
      if (t0 == 0) t0 = t;
      else if (t - t0 > 2000000000ull) return false;
    }
  }
}

// Bounded wait: returns false (and never hangs) if the phase does not
// complete within `limit` suspended polls of at most 1 ms each.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t limit = 1000u) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait_hint(bar, parity, 1000000u)) return true;
  return false;
}

// ---------------------------------------------------------------------------
// cp.async staging of read-only tables (16-byte granules, all in flight at
// once; the hardware wait needs no polling loop)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Copy `bytes` (a multiple of 16, both ends 16-byte aligned) into shared
// memory cooperatively; caller synchronises the block afterwards.
__device__ __forceinline__ void stage_async(void* dst, const void* src, int bytes, int tid,
                                            int nthreads) {
  char* d = static_cast<char*>(dst);
  const char* s = static_cast<const char*>(src);
  for (int off = tid * 16; off < bytes; off += nthreads * 16) cp_async16(d + off, s + off);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start while its predecessor is still running; it must
// call pdl_wait() before touching anything the predecessor writes or reads.
// Without the launch attribute both are no-ops in effect.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Tensor-core helpers (mma.sync m16n8k16 f16 -> f32, movmatrix)
// ---------------------------------------------------------------------------
// Not volatile: the MMA has no side effect beyond its outputs, so the
// compiler may interleave independent accumulator chains.
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4],
                                              uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace tq
