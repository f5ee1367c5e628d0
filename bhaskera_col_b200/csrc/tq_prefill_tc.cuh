// tq_prefill_tc.cuh — device pieces shared by the tcgen05 prefill-attention
// kernels (tq_prefill_tc.cu: 128 query rows per CTA; tq_prefill_tc2.cu: 256):
// MMA issue and descriptors, tensor-memory access, the bounded wait, and the
// decoders that turn packed codes into fp16 K^ / V^ tiles in the 128-byte
// swizzle layout.
//
// Layout conventions: head_dim 128; key tiles of 128 tokens (two pages); an
// operand tile is [64-column half][rows][128 B], 16-byte chunk c of row r at
// sw_chunk(r, c).  K^ is read K-major (B of S = q' K^^T) and V^ MN-major (B of
// O = P V^) from the same physical layout.  Columns stay in the packed orders
// of the page rows: K quad order (k_coord) and V octet order (v_coord).
#pragma once

#include "tq_common.cuh"
#include "tq_internal.h"
#include "tq_tc.cuh"

namespace tq {
namespace pftc {

constexpr int kD = 128;
constexpr int kKeys = 128;                 // keys per tile (two pages)
constexpr uint32_t kHalfBytes = 16384;     // [128 rows][128 B]
constexpr uint32_t kStage = 2 * kHalfBytes;
constexpr float kRescaleBits = 8.f;        // lazy rescale threshold (log2)
constexpr float kLog2e = 1.4426950408889634f;

struct TcPrefillParams {
  const uint8_t* pages;
  PageMap pm;
  int page_bytes, off_v, off_kn, off_vn;
  const __half* rot_h;          // R [128][128] fp16, row-major
  const float* rot;             // R [128][128] fp32, row-major
  const float* kc;
  const float* vc;
  const void* q; int q_dtype; int q_vec; int64_t qs[4];
  void* out; int o_dtype; int o_vec; int64_t os[4];
  int64_t Hkv, g, Tq, n_tokens;
  int hc, pshift;               // heads per CTA; log2(positions per 128-row tile)
  int nqb;
  int pcta;                     // positions per CTA (two-tile kernel)
  int tile_head_step, tile_pos_step;   // tile X's first head / position offset
  float qscale;                 // softmax scale * log2(e)
  int causal;
  int rk, rv;                   // pair-table replication (lanes per copy set)
  const int32_t* kv_start;      // [B] first attended key of each batch row, or NULL
  // residual window: keys n_tokens - W .. n_tokens - 1 come rotated (fp16,
  // [stream][W][128], K quad / V octet order) from wk / wv instead of pages
  const __half* wk;
  const __half* wv;
  int64_t W;
  uint32_t* status;
};

// D (+)= A B with A and B in shared memory (kind::f16: fp16 or bf16 by idesc).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  tc::umma_bf16(d_tmem, a_desc, b_desc, idesc, accumulate);
}

// D (+)= A B with A in tensor memory (lanes = rows, two 16-bit elements per
// column) and B in shared memory.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// MN-major operand in the 128-byte swizzle layout: rows of 64 MN-contiguous
// 16-bit elements (128 B), 8-row groups 1024 B apart (stride byte offset),
// 64-element MN blocks `lbo` bytes apart (leading byte offset).
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// tcgen05.wait::ld that also names the destination registers, so no use of
// them can be scheduled above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :: "memory");
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Scores of keys before `first` or past `last` (indices into this 32-key
// chunk) -> -inf.
__device__ __forceinline__ void mask_keys(uint32_t (&x)[32], int64_t first, int64_t last) {
#pragma unroll
  for (int e = 0; e < 32; ++e)
    if (e > last || e < first) x[e] = 0xFF800000u;
}

// The first key batch row b attends (left padding), >= 0.
__device__ __forceinline__ int64_t row_kstart(const int32_t* kv_start, int64_t b) {
  if (!kv_start) return 0;
  const int v = __ldg(kv_start + b);
  return v < 0 ? 0 : v;
}

// fp16 pair {exp2(a - bias), exp2(b - bias)} (a in the low half): the
// differences rounded to fp16 (|a - bias| < 2^4 carries an error below 2^-7
// in the exponent only for p < 2^-4), then one SFU op for both exponentials.
__device__ __forceinline__ uint32_t exp2_pair(uint32_t a, uint32_t b, uint64_t nbias2) {
  uint32_t h, p;
  asm("{\n .reg .b64 x, y;\n .reg .f32 lo, hi;\n"
      " mov.b64 x, {%1, %2};\n add.rn.f32x2 y, x, %3;\n mov.b64 {lo, hi}, y;\n"
      " cvt.rn.f16x2.f32 %0, hi, lo;\n}"
      : "=r"(h) : "r"(a), "r"(b), "l"(nbias2));
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(p) : "r"(h));
  return p;
}

using tc::tmem_st_x16;

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
               ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// The `rep` copies of pair-table entry e (4 bytes each) at `table`: 16-byte
// stores where the copies come in fours, else one store per copy.
__device__ __forceinline__ void put_pair_entry(uint32_t table, int e, int rep, uint32_t v) {
  const uint32_t at = table + 4u * (uint32_t)(e * rep);
  if (rep >= 4) {
    for (int c = 0; c < rep; c += 4) sts128(at + 4u * (uint32_t)c, make_uint4(v, v, v, v));
  } else {
    for (int c = 0; c < rep; ++c) sts32(at + 4u * (uint32_t)c, v);
  }
}

// Byte offset of 16-byte chunk `c` (0..15, 8 elements each) of row `r` in a
// [2][rows][128 B] swizzled operand.
__device__ __forceinline__ uint32_t sw_chunk(int r, int c) {
  return (uint32_t)((c >> 3) * kHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Coordinate held at position i of a K row (quad order) / V row (octet order).
__device__ __forceinline__ int k_coord(int i) {
  const int t = i >> 5, e = i & 31;
  return 16 * (e >> 2) + 2 * t + (e & 1) + 8 * ((e >> 1) & 1);
}
__device__ __forceinline__ int v_coord(int i) { return (i >> 4) + 8 * (i & 15); }

__device__ __forceinline__ void fail(uint32_t* status, volatile int* abort_flag) {
  *abort_flag = 1;
  atomicOr(status, TQ_DEV_WAIT_TIMEOUT);
}

// Bounded wait (2 s) that also gives up as soon as another role has aborted.
// try_wait without a suspend-time hint (a hinted wait wakes about 0.1 us late,
// more than this kernel's per-tile hand-offs can afford) and a short sleep
// between polls, so waiting warps leave the issue slots to working ones.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity,
                                              volatile int* abort_flag, uint32_t* status) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(32);
    if ((i & 255u) == 255u) {
      if (*abort_flag) return false;
      const uint64_t t = global_ns();
      if (t0 == 0) t0 = t;
      else if (t - t0 > 2000000000ull) break;
    }
  }
  fail(status, abort_flag);
  return false;
}

// 8-element fp16 chunk of a 16-bit source row -> fp16 scaled by s.
__device__ __forceinline__ uint4 scale_chunk(uint4 raw, int dtype, float s) {
  uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float lo, hi;
    if (dtype == TQ_F16) {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      lo = __low2float(h); hi = __high2float(h);
    } else {
      lo = __uint_as_float(w[i] << 16);
      hi = __uint_as_float(w[i] & 0xFFFF0000u);
    }
    o[i] = pack_half2(lo * s, hi * s);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Codes of one 32-position stream (a K quad or a V octet pair): NB words.
template <int NB>
struct Stream { uint32_t w[NB]; };

template <int NB>
__device__ __forceinline__ void load_stream(Stream<NB>& s, const uint8_t* src) {
  if constexpr (NB == 4) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
    s.w[0] = v.x; s.w[1] = v.y; s.w[2] = v.z; s.w[3] = v.w;
  } else if constexpr (NB == 2) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(src));
    s.w[0] = v.x; s.w[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < NB; ++i) s.w[i] = __ldg(reinterpret_cast<const uint32_t*>(src) + i);
  }
}

// Pair p (positions 2p, 2p+1) of a stream of NB-bit codes: a 2*NB-bit index.
template <int NB>
__device__ __forceinline__ uint32_t pair_index(const Stream<NB>& s, int p) {
  const int bo = 2 * NB * p, w = bo >> 5, sh = bo & 31;
  constexpr uint32_t mask = (1u << (2 * NB)) - 1u;
  if (sh + 2 * NB <= 32) return (s.w[w] >> sh) & mask;
  return __funnelshift_r(s.w[w], s.w[w + 1], sh) & mask;
}

// Byte offsets (within a stage, page 0) of the four 16-byte chunks a decoder
// thread writes: chunks 4 part .. 4 part + 3 of row kk.  With the XOR swizzle
// they are (c ^ q) << 4 for one per-thread constant c, so no address math is
// left in the tile loop.
struct ChunkOffsets { uint32_t o[4]; };
__device__ __forceinline__ ChunkOffsets chunk_offsets(int kk, int part) {
  ChunkOffsets r;
#pragma unroll
  for (int q = 0; q < 4; ++q) r.o[q] = sw_chunk(kk, 4 * part + q);
  return r;
}

// Decode a 32-position stream into 4 fp16 chunks (x norm) and store them at
// `tile` + co.o[q].  Plain C++ shared loads and stores (no volatile asm), so
// the compiler can issue every table lookup of a tile ahead of the stores;
// the proxy fence that follows a tile orders the stores before the hand-off.
template <int NB>
__device__ __forceinline__ void decode_stream(const Stream<NB>& s, const unsigned char* lut,
                                              int rep4, __half2 n2, unsigned char* tile,
                                              const ChunkOffsets& co) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t h[4];
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      uint32_t v = *reinterpret_cast<const uint32_t*>(lut + pair_index<NB>(s, 4 * q + pp) * rep4);
      __half2 x = *reinterpret_cast<__half2*>(&v);
      x = __hmul2(x, n2);
      h[pp] = *reinterpret_cast<uint32_t*>(&x);
    }
    *reinterpret_cast<uint4*>(tile + co.o[q]) = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

struct TcParamsView {
  const uint8_t* pool;          // the pages (contiguous streams or a block pool)
  PageMap pm;
  int64_t stream;
  uint32_t* status;             // TQ_DEV_BAD_BLOCK on a block-table entry outside the pool
  int page_bytes, off_v, off_kn, off_vn;
  int kk, part;
  int64_t kend;                 // keys this CTA needs
  int64_t kpacked;              // keys [0, kpacked) are in pages, the rest in the window
  int64_t W;                    // window tokens (rows of the rotated window buffers)
};

// One operand's codes and norms that a decoder thread needs for one tile:
// NR rows (NR / 2 per page: keys kk + (64 / (NR / 2)) * i of each page), K
// quad / V octet pair `part`.
template <int NB, int NR>
struct HalfRegs {
  Stream<NB> c[NR];
  uint32_t n[NR];               // fp16 norm bits
};

template <int NB, int NR>
__device__ __forceinline__ void load_half(HalfRegs<NB, NR>& t, const TcParamsView& pv, int j,
                                          int off_codes, int off_norm) {
  constexpr int RPP = NR / 2, STEP = 64 / RPP;
  const uint8_t* pgs[2];
  const int64_t kpend = tmin<int64_t>(pv.kend, pv.kpacked);   // needed keys held in pages
#pragma unroll
  for (int pgi = 0; pgi < 2; ++pgi) {
    pgs[pgi] = pv.pool;
    if ((int64_t)j * kKeys + pgi * 64 < kpend) {        // the page holds needed keys
      bool ok;
      const int64_t ps = page_slot(pv.pm, pv.stream, 2 * (int64_t)j + pgi, ok);
      if (!ok) atomicOr(pv.status, TQ_DEV_BAD_BLOCK);
      pgs[pgi] = pv.pool + ps * (int64_t)pv.page_bytes;
    }
  }
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int pgi = r / RPP, key_in_page = pv.kk + STEP * (r % RPP);
    const int64_t key = (int64_t)j * kKeys + pgi * 64 + key_in_page;
    if (key < kpend) {
      const uint8_t* pg = pgs[pgi];
      load_stream<NB>(t.c[r], pg + off_codes + key_in_page * (16 * NB) + pv.part * (4 * NB));
      t.n[r] = __ldg(reinterpret_cast<const unsigned short*>(pg + off_norm) + key_in_page);
    } else {
#pragma unroll
      for (int i = 0; i < NB; ++i) t.c[r].w[i] = 0u;
      t.n[r] = 0u;
    }
  }
}

// Decode the NR rows of one operand tile into the stage at `tile` (row
// 64 pgi + kk + STEP i sits (64 pgi + STEP i) * 128 bytes below row kk, with
// the same swizzle).
template <int NB, int NR>
__device__ __forceinline__ void decode_half(const HalfRegs<NB, NR>& t, const unsigned char* lut,
                                            int rep4, unsigned char* tile, const ChunkOffsets& co) {
  constexpr int RPP = NR / 2, STEP = 64 / RPP;
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const uint32_t n2 = t.n[r] * 0x10001u;
    decode_stream<NB>(t.c[r], lut, rep4, *reinterpret_cast<const __half2*>(&n2),
                      tile + ((r / RPP) * 64 + STEP * (r % RPP)) * 128, co);
  }
}


// Rows of tile j that lie in the residual window: copy the thread's 32
// positions (4 chunks) of the rotated fp16 row straight into the tile, over
// what decode_half wrote there (zeros: such rows load no codes).
template <int NR>
__device__ __forceinline__ void window_half(const TcParamsView& pv, int j, const __half* wbuf,
                                            unsigned char* tile, const ChunkOffsets& co) {
  constexpr int RPP = NR / 2, STEP = 64 / RPP;
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int pgi = r / RPP, kin = pv.kk + STEP * (r % RPP);
    const int64_t key = (int64_t)j * kKeys + pgi * 64 + kin;
    if (key >= pv.kpacked && key < pv.kend) {
      const uint4* src = reinterpret_cast<const uint4*>(
          wbuf + ((pv.stream * pv.W + (key - pv.kpacked)) * kD + pv.part * 32));
      unsigned char* row = tile + (pgi * 64 + STEP * (r % RPP)) * 128;
#pragma unroll
      for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(row + co.o[q]) = __ldg(src + q);
    }
  }
}

// Does tile j hold any window key this CTA needs?
__device__ __forceinline__ bool tile_has_window(const TcParamsView& pv, int j) {
  return pv.W > 0 && (int64_t)(j + 1) * kKeys > pv.kpacked && (int64_t)j * kKeys < pv.kend;
}

}  // namespace pftc

// The 256-row kernel (tq_prefill_tc2.cu): TQ_OK when it ran, 1 when no
// variant exists for (kb, vb), or an error.
int launch_prefill_tc2(const pftc::TcPrefillParams& base, int kb, int vb, int64_t B, int64_t Hq,
                       cudaStream_t st);

}  // namespace tq
