// tq_decode.cu — single-token GQA decode attention straight off the packed
// TurboQuant pages.
//
// Replaces: HF attention (torch SDPA with GQA repeat) over the dequantised
// K/V that TurboQuantKVCache.update returns (aditya25058/Bhaskera_col
// src/bhaskera/inference/kv_cache.py:483-488, 580-589; engine.py:389).
//
// Math.  With R the layer rotation and k_t = n_t (c[idx_t] R), the score is
//   <q, k_t> = n_t <q R^T, c[idx_t]>,
// so the query is rotated once (prep_kernel) and keys are never
// un-rotated.  Likewise o = sum_t p_t n_t (c_v[idx_t] R) = (sum_t p_t n_t
// c_v[idx_t]) R: values are accumulated in the rotated basis and un-rotated
// once per head in merge_kernel.  The optional QJL term adds
// gamma_t * alpha * <S q_rot, sign_t>.
//
// Kernels per call:
//   prep_kernel    q_rot, S q_rot -> fp16 fragments (scale * log2e folded in);
//                  in a decode step also the append of the new token
//   decode_kernel  persistent, one CTA per SM; each of its page groups (a
//                  work unit) owns a contiguous range of the flattened
//                  (stream, page) space.  A producer warp streams 64-token
//                  pages into shared memory with bulk async copies (no
//                  multicast) through full/empty mbarriers; the group's four
//                  consumer warps take pages in pairs, 32 tokens per warp,
//                  dequantise codes straight into mma.sync fragments through
//                  lane-replicated pair lookup tables, and run an online
//                  softmax.  The self-fed variant (uniform batch on contiguous
//                  pages) has no producer warp: consumer threads issue the
//                  copies themselves.  One partial (m, l, O_rot) per
//                  (stream, head, work unit) touched.
//   merge_kernel   combines the partials of each (stream, head), attends the
//                  full-precision window, un-rotates, writes the output.
#include "tq_common.cuh"
#include "tq_internal.h"
#include "tq_vec.cuh"

#include <math.h>

namespace tq {

constexpr int kTileWarps = 4;     // warps of a page group (two per page, 32 tokens each)
// dynamic shared memory a decode CTA may take: the 227 KB opt-in limit less
// 1 KB for the kernel's static shared memory
constexpr int kSmemBudget = 226 * 1024;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -INFINITY;
// The decode's softmax bias runs this far (log2 units) above the running max,
// so the max is reduced across a warp only when a score passes it.
constexpr float kLazyBits = 8.f;

// Which pages a decode walks.  Stream s owns the compacted page range
// [start(s), start(s + 1)): s * Pv for a uniform batch, and for a ragged one
// (per-row token counts) the prefix sums the query preparation lays out.
// Work unit u (a page group of a decode CTA) takes compacted pages
// [u * Q, (u + 1) * Q).
struct PageLayout {
  int64_t S, Pv, T, Q;    // streams, pages and tokens per stream (bounds), pages per unit
  int hkv;                // streams per batch row
  int64_t nid;            // partial-result ids per head chunk: work units + S
  const int32_t* lens;    // [B] tokens of each batch row; NULL: uniform (T each)
  int32_t* cum;           // [S + 1] ragged: first compacted page of each stream
  int32_t* rq;            // ragged: pages per unit
  const int32_t* kstart;  // [B] first attended position of each batch row (left padding); NULL: 0
};

// A ragged layout opens every non-empty stream with this many placeholder
// pages: the cost of a stream boundary (the group drains, combines and
// starts the next stream, ~3.5 us, about four pages) counted as work, so the
// units over many short requests take fewer real pages.  Placeholders are
// never fetched or computed; producer and consumers skip them alike.
constexpr int kSegPages = 4;

__device__ __forceinline__ int64_t lay_start(const PageLayout& L, int64_t s) {
  return L.lens ? (int64_t)__ldcg(L.cum + s) : s * L.Pv;
}

__device__ __forceinline__ int lay_tokens(const PageLayout& L, int64_t s) {
  if (!L.lens) return (int)L.T;
  const int64_t n = __ldg(L.lens + s / L.hkv);
  return (int)(n < 0 ? 0 : n > L.T ? L.T : n);
}

// First position stream s attends (left padding), >= 0.
__device__ __forceinline__ int lay_kstart(const PageLayout& L, int64_t s) {
  if (!L.kstart) return 0;
  const int v = __ldg(L.kstart + s / L.hkv);
  return v < 0 ? 0 : v;
}

// The stream owning compacted page x (< cum[S]): the largest s with
// cum[s] <= x, found by a 32-way search of the whole warp (two rounds up to
// 1,024 streams).  Invariant: cum[lo] <= x < cum[hi] (cum[S] is the total).
__device__ __forceinline__ int64_t find_stream(const int32_t* cum, int64_t S, int64_t x, int lane) {
  int64_t lo = 0, hi = S;
  while (hi - lo > 1) {
    const int64_t step = (hi - lo + 31) / 32;
    const int64_t i = lo + lane * step;
    const bool le = i < hi && (int64_t)__ldcg(cum + i) <= x;
    const unsigned m = __ballot_sync(0xffffffffu, le);
    lo += (31 - __clz(m)) * step;
    hi = tmin<int64_t>(hi, lo + step);
  }
  return lo;
}

struct DecodeParams {
  const uint8_t* pages;
  PageMap pm;
  PageLayout lay;
  int nch;
  const uint32_t* qf;    // [S][nch][8][D/2] half2
  const uint32_t* sqf;   // [S][nch][8][D/2] half2
  const float* kc;
  const float* vc;
  // partial results of segment (work unit u, stream s) under id u + s: the
  // id grows along every unit's walk and from one unit to the next, so ids
  // of different segments never meet
  float* part_m;         // [nch][nid][8]
  float* part_l;
  float* part_o;         // [nch][nid][8][D]
  uint32_t* status;
};

__host__ __device__ constexpr int align128(int x) { return (x + 127) & ~127; }
__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }

// ---------------------------------------------------------------------------
// lookup tables.  Pair tables (2 * bits <= 8): entry e = c_lo | c_hi << bits
// holds half2(c[c_lo], c[c_hi]), replicated per lane so lane l reads bank l:
// byte address (e << 7) | (lane << 2).  Wider codes use a plain fp16 table.
// ---------------------------------------------------------------------------
template <int BITS>
struct Lut {
  static constexpr bool kPair = 2 * BITS <= 8;
  static constexpr int kBytes = kPair ? (1 << (2 * BITS)) * 128 : (1 << BITS) * 2;
};

template <int BITS>
__device__ __forceinline__ void build_lut(unsigned char* base, const float* cent, int tid,
                                          int nthreads) {
  if constexpr (Lut<BITS>::kPair) {
    uint32_t* lut = reinterpret_cast<uint32_t*>(base);
    constexpr int E = 1 << (2 * BITS);
    for (int i = tid; i < E * 32; i += nthreads) {
      const int e = i >> 5;
      lut[i] = pack_half2(__ldg(cent + (e & ((1 << BITS) - 1))), __ldg(cent + (e >> BITS)));
    }
  } else {
    __half* h = reinterpret_cast<__half*>(base);
    for (int i = tid; i < (1 << BITS); i += nthreads) h[i] = __float2half_rn(__ldg(cent + i));
  }
}

// Byte offset (field << 7) | lane4 of the W-bit field starting at bit o of w[].
template <int W, int NW>
__device__ __forceinline__ uint32_t field_addr(const uint32_t (&w)[NW], int o, uint32_t lane4) {
  const int wi = o >> 5, sh = o & 31;
  uint32_t x;
  if (sh + W <= 32 || wi + 1 >= NW) {
    x = sh >= 7 ? (w[wi] >> (sh - 7)) : (w[wi] << (7 - sh));
  } else {
    x = __funnelshift_r(w[wi], w[wi + 1], sh) << 7;
  }
  return (x & (((1u << W) - 1u) << 7)) | lane4;
}

template <int NW>
__device__ __forceinline__ uint32_t getbits(const uint32_t (&w)[NW], int o, int n) {
  const int wi = o >> 5, sh = o & 31;
  uint32_t v;
  if (sh + n <= 32 || wi + 1 >= NW) v = w[wi] >> sh;
  else v = __funnelshift_r(w[wi], w[wi + 1], sh);
  return v & ((1u << n) - 1u);
}

// Loads from a lookup table in (static) shared memory; with a static table
// the table's address folds into the load's immediate offset.
__device__ __forceinline__ uint32_t lds32(const unsigned char* base, uint32_t byte_off) {
  return *reinterpret_cast<const uint32_t*>(base + byte_off);
}
__device__ __forceinline__ uint32_t lds16(const unsigned char* base, uint32_t byte_off) {
  return *reinterpret_cast<const unsigned short*>(base + byte_off);
}

// Load NBITS bits starting at bit `bit_off` of a 4-byte aligned shared row.
template <int NBITS, bool ALIGNED>
__device__ __forceinline__ void load_bits(const uint8_t* row, int bit_off,
                                          uint32_t (&w)[(NBITS + 31) / 32]) {
  constexpr int NW = (NBITS + 31) / 32;
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row) + (bit_off >> 5);
  if constexpr (ALIGNED && NW % 4 == 0) {
#pragma unroll
    for (int i = 0; i < NW; i += 4) {
      uint4 v = *reinterpret_cast<const uint4*>(p + i);
      w[i] = v.x; w[i + 1] = v.y; w[i + 2] = v.z; w[i + 3] = v.w;
    }
  } else if constexpr (ALIGNED && NW % 2 == 0) {
#pragma unroll
    for (int i = 0; i < NW; i += 2) {
      uint2 v = *reinterpret_cast<const uint2*>(p + i);
      w[i] = v.x; w[i + 1] = v.y;
    }
  } else if constexpr (ALIGNED) {
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = p[i];
  } else {
    const int sh = bit_off & 31;
    uint32_t prev = p[0];
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      uint32_t nxt = p[i + 1];
      w[i] = sh ? __funnelshift_r(prev, nxt, sh) : prev;
      prev = nxt;
    }
  }
}

// +-1 half2 from the sign bits at positions pe (low half) and po (high half);
// bit set <=> +1.
__device__ __forceinline__ uint32_t sign_pair(uint32_t w, int pe, int po) {
  if (po == pe + 16 && pe <= 15) return ((w << (15 - pe)) & 0x80008000u) ^ 0xBC00BC00u;
  uint32_t e = (w >> pe) & 1u, o = (w >> po) & 1u;
  return 0xBC00BC00u ^ ((e << 15) | (o << 31));
}

__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// The named barrier of page group `grp` (ids 1..NG, constant in each branch
// so the kernel reserves NG + 1 barriers, not all sixteen).
template <int NG>
__device__ __forceinline__ void group_bar(int grp, int count) {
  static_assert(NG >= 1 && NG <= 4, "page groups");
  if constexpr (NG == 1) {
    named_bar(1, count);
  } else {
    if (grp == 0) named_bar(1, count);
    else if (NG == 2 || grp == 1) named_bar(2, count);
    else if (NG == 3 || grp == 2) named_bar(3, count);
    else named_bar(4, count);
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// ---------------------------------------------------------------------------
// decode kernel
// ---------------------------------------------------------------------------
template <int D, int KB, int VB, bool QJL>
struct Dec {
  // page geometry (compile time; matches make_geom)
  static constexpr int KROW = D * KB / 8, VROW = D * VB / 8, QROW = QJL ? D / 8 : 0;
  static constexpr int OFF_V = 64 * KROW, OFF_Q = OFF_V + 64 * VROW;
  static constexpr int OFF_KN = OFF_Q + 64 * QROW, OFF_VN = OFF_KN + 128, OFF_KR = OFF_VN + 128;
  static constexpr int PAGE = OFF_KR + (QJL ? 128 : 0);
  static constexpr int PB = align128(PAGE);
  // static shared memory: the K table (aliased by the combine scratch) and,
  // when both fit, the V table.  Dynamic: [V table] [stages] [barriers]
  // (FAST: [table] [stages] [barriers] [combine scratch]).
  // K4 with V2 / V4 at D128: one 64 KB dynamic table region, 256 rows of
  // 256 B (one row per code byte): bytes 0-127 the K pair entry for each of
  // 32 lanes, bytes 128-255 the V entry (V4: pair for 32 lanes; V2: quad of
  // 8 B for 16 lanes).  A lookup address is (byte << 8) | lane offset: one
  // byte permute.  Such a CTA owns its SM: 12 consumer warps in three groups
  // of four take every third page, so one table serves as many warps as
  // three CTAs of the other variants do, and the combine scratch has its own
  // region (no table rebuild where a stream ends, as ragged batches often do).
  static constexpr bool FAST = D == 128 && KB == 4 && (VB == 2 || VB == 4);
  static constexpr int NCW = FAST ? 12 : 4;            // consumer warps
  static constexpr int NG = NCW / kTileWarps;          // page groups
  static constexpr int THREADS = 32 * (NCW + 1);       // + one producer warp
  static constexpr int MINB = FAST ? 1 : 3;            // CTAs per SM
  // stages per page group (pages go in pairs): 4, or 3 where four do not fit
  // beside the FAST table and its combine scratch
  static constexpr int SG =
      (FAST && 65536 + NG * 4 * PB + 2 * NG * 4 * 8 + 128 + NCW * (16 + 8 * D) * 4 > kSmemBudget)
          ? 3 : 4;
  static constexpr int STAGES = NG * SG;
  static constexpr int COMB = NCW * (16 + 8 * D) * 4;
  static constexpr int FLUT = 65536;
  static constexpr int REGION0 = FAST ? 128 : align128(cmax(Lut<KB>::kBytes, COMB));
  static constexpr bool VSTATIC = FAST || REGION0 + Lut<VB>::kBytes <= 45 * 1024;
  static constexpr int LUTV_STATIC = (VSTATIC && !FAST) ? Lut<VB>::kBytes : 16;
  static constexpr int LUTV = 0;   // offset of the V table in the dynamic region
  static constexpr int STAGE0 = FAST ? FLUT : VSTATIC ? 0 : align128(Lut<VB>::kBytes);
  static constexpr int BARS = STAGE0 + STAGES * PB;
  static constexpr int COMB_OFF = align128(BARS + 2 * STAGES * 8);
  static constexpr int SMEM = FAST ? COMB_OFF + COMB : BARS + 2 * STAGES * 8;
  static_assert(SMEM <= kSmemBudget, "shared memory");
};

// The K4 / V2|V4 table region (see Dec::FAST): rows [r0, r1) of 256 B, one
// 16-byte chunk per thread and step (consecutive threads, consecutive chunks).
template <int VB>
__device__ __forceinline__ void build_fast_lut(unsigned char* base, const float* kc,
                                               const float* vc, int r0, int r1, int tid,
                                               int nthreads) {
  uint4* L = reinterpret_cast<uint4*>(base);
  for (int i = r0 * 16 + tid; i < r1 * 16; i += nthreads) {
    const int e = i >> 4, c = i & 15;
    uint4 val;
    if (c < 8) {
      const uint32_t k = pack_half2(__ldg(kc + (e & 15)), __ldg(kc + (e >> 4)));
      val = make_uint4(k, k, k, k);
    } else if constexpr (VB == 4) {
      const uint32_t v = pack_half2(__ldg(vc + (e & 15)), __ldg(vc + (e >> 4)));
      val = make_uint4(v, v, v, v);
    } else {
      // byte e = a0 | a1 << 2 | b0 << 4 | b1 << 6 (codes of tokens a, b at
      // two positions): half2(c[a0], c[b0]) then half2(c[a1], c[b1])
      const uint32_t v0 = pack_half2(__ldg(vc + (e & 3)), __ldg(vc + ((e >> 4) & 3)));
      const uint32_t v1 = pack_half2(__ldg(vc + ((e >> 2) & 3)), __ldg(vc + (e >> 6)));
      val = make_uint4(v0, v1, v0, v1);
    }
    L[i] = val;
  }
}

// (byte b of x) << 8 | low byte of lane_off: the address of a fast-table
// lookup, in one byte permute (the other bytes of lane_off are zero).
__device__ __forceinline__ uint32_t fast_addr(uint32_t x, uint32_t lane_off, int b) {
  return __byte_perm(x, lane_off, 0x5504u | ((uint32_t)b << 4));
}

__device__ __forceinline__ uint2 lds64(const unsigned char* base, uint32_t byte_off) {
  return *reinterpret_cast<const uint2*>(base + byte_off);
}

// SELF (head_dim-128 K4 / V2|V4 kernels, uniform batches on contiguous
// pages): no producer warp.  A page group's first thread fills its ring and
// the first warp of each page's warp pair refills that page's stage with the
// page SG later, once both warps have released it; page addresses follow from
// the page index alone.  Without the 13th warp the compiler may give each
// thread up to 168 registers instead of 128 (13 warps put four on one
// scheduler): 2.7 % faster on the Mixtral layer.
template <int D, int KB, int VB, bool QJL, bool SELF = false>
__global__ void __launch_bounds__(SELF ? 32 * Dec<D, KB, VB, QJL>::NCW : Dec<D, KB, VB, QJL>::THREADS,
                                  Dec<D, KB, VB, QJL>::MINB)
decode_kernel(DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  using G = Dec<D, KB, VB, QJL>;
  constexpr int NJ = D / 16;                 // 16-coordinate chunks
  constexpr int KQB = (D / 4) * KB;          // bits per K quad
  constexpr int KQW = (KQB + 31) / 32;
  constexpr bool KQA = (KQB % 32) == 0;
  constexpr int VOB = (D / 8) * VB;          // bits per V octet
  constexpr int VOW = (VOB + 31) / 32;
  constexpr bool VOA = (VOB % 32) == 0;
  constexpr int QQB = D / 4;                 // QJL bits per quad
  constexpr int QQW = (QQB + 31) / 32;
  constexpr int SP = (D / 8) < 16 ? (D / 8) : 16;
  constexpr bool VINTER = Lut<VB>::kPair && (32 % VB == 0) && VOA;

  __shared__ __align__(128) unsigned char s_lut0[G::REGION0];
  __shared__ __align__(128) unsigned char s_lutv_static[G::LUTV_STATIC];
  unsigned char* stages = smem + G::STAGE0;
  unsigned char* lutk = G::FAST ? smem : s_lut0;
  unsigned char* lutv = G::FAST ? smem : G::VSTATIC ? s_lutv_static : smem + G::LUTV;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::BARS);
  constexpr int kStages = G::STAGES;
  constexpr int kConsumerWarps = G::NCW;
  uint64_t* empty = full + kStages;
  __shared__ int s_abort;
  __shared__ int s_issued[SELF ? kStages : 1];  // SELF: copies issued into each stage
  static_assert(!SELF || G::FAST, "self-fed kernels are the FAST variants");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hc = blockIdx.y;
  const PageLayout& L = p.lay;
  constexpr int NCT = 32 * kConsumerWarps;   // consumer threads

  if (tid == 0) {
    s_abort = 0;
    if constexpr (SELF)
      for (int s = 0; s < kStages; ++s) s_issued[s] = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kTileWarps / 2);   // the two warps that take a page
    }
    fence_mbar_init();
  }
  pdl_launch_dependents();
  if (warp < kConsumerWarps) {
    if constexpr (G::FAST) {
      build_fast_lut<VB>(smem, p.kc, p.vc, 0, 256, tid, NCT);
    } else {
      build_lut<KB>(lutk, p.kc, tid, NCT);
      build_lut<VB>(lutv, p.vc, tid, NCT);
    }
  }
  __syncthreads();
  pdl_wait();   // pages, query fragments and a ragged layout come from the preceding kernels

  // Work unit u = blockIdx.x * NG + g, served by page group g (its four
  // consumer warps and producer lane g), takes compacted pages
  // [u * Q, (u + 1) * Q).  Each group walks and combines its own streams, so
  // where one group's stream ends the other groups keep working (a CTA over
  // many short requests of a ragged batch would otherwise stop all twelve
  // warps at every stream boundary).  unit_range runs on whole warps (the
  // stream search is warp-cooperative) and is warp-uniform.
  const int64_t Q = L.lens ? (int64_t)__ldcg(L.rq) : L.Q;
  const int64_t total = L.lens ? (int64_t)__ldcg(L.cum + L.S) : L.S * L.Pv;
  auto unit_range = [&](int g, int64_t& u0, int& n, int64_t& sf) {
    const int64_t u = (int64_t)blockIdx.x * G::NG + g;
    u0 = u * Q;
    n = (int)tmax<int64_t>(0, tmin<int64_t>(u0 + Q, total) - u0);
    sf = 0;                                      // the stream of page u0
    if (n > 0) sf = L.lens ? find_stream(L.cum, L.S, u0, lane) : u0 / L.Pv;
  };

  // ------------------------------------------------------------ producer
  // Lane g feeds page group g (its unit's pages in order) through its own
  // ring of SG stages, so a slow group never holds back the others' pages.
  if (warp == kConsumerWarps) {
    int64_t gp0 = 0, s_first = 0;
    int npages = 0;
    for (int g = 0; g < G::NG; ++g) {
      int64_t a, sf;
      int n;
      unit_range(g, a, n, sf);
      if (lane == g) { gp0 = a; npages = n; s_first = sf; }
    }
    if (lane < G::NG) {
      const int gr = lane;
      int issued = 0;
      // The lane's pages come in increasing order: walk the streams with the
      // next stream's start held in a register (a load only when the walk
      // crosses into the next stream; gpi < total, so it stops before S),
      // and load each page's table entry one page ahead, before the wait
      // for its stage, so the lookup latency hides behind that wait.
      int64_t sp = s_first, sp0 = lay_start(L, sp), nx = lay_start(L, sp + 1);
      const int cph = L.lens ? kSegPages : 0;
      // false for a placeholder page; else the page's table entry in e
      auto locate = [&](int64_t gpi, int64_t& e) {
        while (nx <= gpi) {
          ++sp;
          sp0 = nx;
          nx = lay_start(L, sp + 1);
        }
        const int64_t pg = gpi - sp0 - cph;
        if (pg < 0) return false;
        e = page_entry(p.pm, sp, pg);
        return true;
      };
      int64_t next = 0;
      bool next_real = npages > 0 && locate(gp0, next);
      int kr = 0;                                // real pages issued: the ring position
      for (int k = 0; k < npages; ++k) {
        const int64_t cur = next;
        const bool real = next_real;
        if (k + 1 < npages) next_real = locate(gp0 + k + 1, next);
        if (!real) continue;
        const int st = gr * G::SG + kr % G::SG;
        if (kr >= G::SG && !s_abort) {
          if (!mbar_wait_poll(&empty[st], (uint32_t)(((kr / G::SG) - 1) & 1))) {
            atomicOr(p.status, TQ_DEV_WAIT_TIMEOUT);
            s_abort = 1;
          }
        }
        if (s_abort) break;
        const bool pok = entry_ok(p.pm, cur);
        if (!pok) atomicOr(p.status, TQ_DEV_BAD_BLOCK);
        const int64_t ps = pok ? cur : 0;
        const uint8_t* src = p.pages + ps * (int64_t)G::PAGE;
        mbar_expect_tx(&full[st], (uint32_t)G::PAGE);
        bulk_g2s(stages + st * G::PB, src, (uint32_t)G::PAGE, &full[st]);
        issued = ++kr;
      }
      if (s_abort) {   // never leave with a copy still writing shared memory
        for (int k = tmax(0, issued - G::SG); k < issued; ++k)
          mbar_wait_bounded(&full[gr * G::SG + k % G::SG], (uint32_t)((k / G::SG) & 1), 16u);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  // A page group's four warps take the unit's pages two at a time: warps 0
  // and 1 the first page of the pair, warps 2 and 3 the second, each warp 32
  // tokens (two 16-token tiles).  Two tiles per warp give every MMA chain a
  // twin to interleave with and let one max reduction serve 32 tokens.
  const int gq = lane >> 2, tq = lane & 3;
  const uint32_t lane4 = (uint32_t)lane << 2;
  uint32_t qf[NJ][2], sqf[NJ][2];
  float O[NJ][4];
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;

  auto reset_state = [&]() {
#pragma unroll
    for (int i = 0; i < NJ; ++i) O[i][0] = O[i][1] = O[i][2] = O[i][3] = 0.f;
    m0 = m1 = kNegInf; l0 = l1 = 0.f;
  };
  auto load_q = [&](int64_t s) {
    const uint32_t* qb = p.qf + ((s * p.nch + hc) * 8 + gq) * (D / 2);
    const uint32_t* sb = p.sqf + ((s * p.nch + hc) * 8 + gq) * (D / 2);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      qf[j][0] = __ldg(qb + 8 * j + tq);
      qf[j][1] = __ldg(qb + 8 * j + tq + 4);
      if constexpr (QJL) {
        sqf[j][0] = __ldg(sb + 8 * j + tq);
        sqf[j][1] = __ldg(sb + 8 * j + tq + 4);
      }
    }
  };
  reset_state();

  const int tw = warp % kTileWarps;              // warp of the page group
  const int half = tw >> 1;                      // 0: first page of a pair, 1: second
  const int wt0 = (tw & 1) * 32;                 // the warp's first token in its page
  const int grp = warp / kTileWarps;             // page group: serves unit blockIdx.x * NG + grp
  constexpr int GT = 32 * kTileWarps;            // threads of a page group
  const int gtid = tid - grp * GT;
  const int64_t unit = (int64_t)blockIdx.x * G::NG + grp;
  int64_t gp0, s_first;
  int npages;
  unit_range(grp, gp0, npages, s_first);
  // SELF: page g of the flattened (stream, page) space of a uniform batch on
  // contiguous pages (no placeholders, no block table)
  auto page_addr = [&](int64_t g) {
    const int64_t sp = g / L.Pv;
    return p.pages + (sp * p.pm.pps + (g - sp * L.Pv)) * (int64_t)G::PAGE;
  };
  auto issue = [&](int stg, int64_t g) {
    mbar_expect_tx(&full[stg], (uint32_t)G::PAGE);
    bulk_g2s(stages + stg * G::PB, page_addr(g), (uint32_t)G::PAGE, &full[stg]);
    ++s_issued[stg];
  };
  if constexpr (SELF) {
    if (gtid == 0)
      for (int k = 0; k < G::SG && k < npages; ++k) issue(grp * G::SG + k, gp0 + k);
  }

  // scores of one 16-token tile (rows r0, r0 + 8 of the page) for the lane's
  // two heads, norms applied; K and QJL fragments dequantised straight from
  // the packed rows
  auto tile_scores = [&](const uint8_t* pgb, int r0, float (&sc)[4]) {
    const int r1 = r0 + 8;
    uint32_t wk0[KQW], wk1[KQW];
    load_bits<KQB, KQA>(pgb + r0 * G::KROW, tq * KQB, wk0);
    load_bits<KQB, KQA>(pgb + r1 * G::KROW, tq * KQB, wk1);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float acc2[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t wq0[QQW], wq1[QQW];
    if constexpr (QJL) {
      load_bits<QQB, (QQB % 32) == 0>(pgb + G::OFF_Q + r0 * G::QROW, tq * QQB, wq0);
      load_bits<QQB, (QQB % 32) == 0>(pgb + G::OFF_Q + r1 * G::QROW, tq * QQB, wq1);
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      uint32_t a[4];
      const int o0 = (4 * j) * KB, o1 = (4 * j + 2) * KB;   // quad entries 4j.., 4j+2..
      if constexpr (G::FAST) {
        // pair bytes 2j and 2j + 1 of the quad
        const int wi = j >> 1, b0 = 2 * (j & 1);
        a[0] = lds32(smem, fast_addr(wk0[wi], lane4, b0));
        a[1] = lds32(smem, fast_addr(wk1[wi], lane4, b0));
        a[2] = lds32(smem, fast_addr(wk0[wi], lane4, b0 + 1));
        a[3] = lds32(smem, fast_addr(wk1[wi], lane4, b0 + 1));
      } else if constexpr (Lut<KB>::kPair) {
        a[0] = lds32(lutk, field_addr<2 * KB>(wk0, o0, lane4));
        a[1] = lds32(lutk, field_addr<2 * KB>(wk1, o0, lane4));
        a[2] = lds32(lutk, field_addr<2 * KB>(wk0, o1, lane4));
        a[3] = lds32(lutk, field_addr<2 * KB>(wk1, o1, lane4));
      } else {
        a[0] = lds16(lutk, getbits(wk0, o0, KB) << 1) | (lds16(lutk, getbits(wk0, o0 + KB, KB) << 1) << 16);
        a[1] = lds16(lutk, getbits(wk1, o0, KB) << 1) | (lds16(lutk, getbits(wk1, o0 + KB, KB) << 1) << 16);
        a[2] = lds16(lutk, getbits(wk0, o1, KB) << 1) | (lds16(lutk, getbits(wk0, o1 + KB, KB) << 1) << 16);
        a[3] = lds16(lutk, getbits(wk1, o1, KB) << 1) | (lds16(lutk, getbits(wk1, o1 + KB, KB) << 1) << 16);
      }
      mma_f16_16816(acc, a, qf[j][0], qf[j][1]);
      if constexpr (QJL) {
        uint32_t b[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int pr = 2 * j + h;                 // pair index in the quad
          const int ch = pr / SP, pin = pr % SP;
          const int pe = ch * 2 * SP + pin, po = pe + SP;
          const int wi = pe >> 5;
          b[2 * h + 0] = sign_pair(wq0[wi], pe & 31, po - (wi << 5));
          b[2 * h + 1] = sign_pair(wq1[wi], pe & 31, po - (wi << 5));
        }
        mma_f16_16816(acc2, b, sqf[j][0], sqf[j][1]);
      }
    }
    const __half* kn = reinterpret_cast<const __half*>(pgb + G::OFF_KN);
    const float n0 = __half2float(kn[r0]), n1 = __half2float(kn[r1]);
    sc[0] = acc[0] * n0; sc[1] = acc[1] * n0; sc[2] = acc[2] * n1; sc[3] = acc[3] * n1;
    if constexpr (QJL) {
      const __half* kr = reinterpret_cast<const __half*>(pgb + G::OFF_KR);
      const float g0 = __half2float(kr[r0]), g1 = __half2float(kr[r1]);
      sc[0] = fmaf(acc2[0], g0, sc[0]); sc[1] = fmaf(acc2[1], g0, sc[1]);
      sc[2] = fmaf(acc2[2], g1, sc[2]); sc[3] = fmaf(acc2[3], g1, sc[3]);
    }
  };

  // O^T += V^T P' for one tile (rows t0r = tile start + 2 tq ...), P' the
  // B fragments of the tile's probabilities times ||v||
  auto tile_pv = [&](const uint8_t* pgb, int tile0, uint32_t pb0, uint32_t pb1) {
    const int t0r = tile0 + 2 * tq;
    uint32_t wa[VOW], wb[VOW], wc[VOW], wd[VOW];
    load_bits<VOB, VOA>(pgb + G::OFF_V + (t0r + 0) * G::VROW, gq * VOB, wa);
    load_bits<VOB, VOA>(pgb + G::OFF_V + (t0r + 1) * G::VROW, gq * VOB, wb);
    load_bits<VOB, VOA>(pgb + G::OFF_V + (t0r + 8) * G::VROW, gq * VOB, wc);
    load_bits<VOB, VOA>(pgb + G::OFF_V + (t0r + 9) * G::VROW, gq * VOB, wd);
    if constexpr (G::FAST && VB == 2) {
      // bytes of lo (hi): codes at positions 4k, 4k+1 (4k+2, 4k+3) of token
      // a in the low nibble and of token b in the high nibble
      const uint32_t lab = (wa[0] & 0x0F0F0F0Fu) | ((wb[0] << 4) & 0xF0F0F0F0u);
      const uint32_t hab = ((wa[0] >> 4) & 0x0F0F0F0Fu) | (wb[0] & 0xF0F0F0F0u);
      const uint32_t lcd = (wc[0] & 0x0F0F0F0Fu) | ((wd[0] << 4) & 0xF0F0F0F0u);
      const uint32_t hcd = ((wc[0] >> 4) & 0x0F0F0F0Fu) | (wd[0] & 0xF0F0F0F0u);
      const uint32_t lane_v = 128u + ((uint32_t)(lane & 15) << 3);
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        const uint2 eab = lds64(smem, fast_addr((i2 & 1) ? hab : lab, lane_v, i2 >> 1));
        const uint2 ecd = lds64(smem, fast_addr((i2 & 1) ? hcd : lcd, lane_v, i2 >> 1));
        const uint32_t a[4] = {eab.x, eab.y, ecd.x, ecd.y};
        mma_f16_16816(O[i2], a, pb0, pb1);
      }
    } else if constexpr (G::FAST && VB == 4) {
      // per word: byte k of lo (hi) = code at position 2k (2k+1) of token a,
      // and of token b in the high nibble
      uint32_t lab[2], hab[2], lcd[2], hcd[2];
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        lab[x] = (wa[x] & 0x0F0F0F0Fu) | ((wb[x] << 4) & 0xF0F0F0F0u);
        hab[x] = ((wa[x] >> 4) & 0x0F0F0F0Fu) | (wb[x] & 0xF0F0F0F0u);
        lcd[x] = (wc[x] & 0x0F0F0F0Fu) | ((wd[x] << 4) & 0xF0F0F0F0u);
        hcd[x] = ((wc[x] >> 4) & 0x0F0F0F0Fu) | (wd[x] & 0xF0F0F0F0u);
      }
      const uint32_t lane_v = 128u + lane4;
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        const int x = i2 >> 2, k = i2 & 3;
        const uint32_t a[4] = {lds32(smem, fast_addr(lab[x], lane_v, k)),
                               lds32(smem, fast_addr(hab[x], lane_v, k)),
                               lds32(smem, fast_addr(lcd[x], lane_v, k)),
                               lds32(smem, fast_addr(hcd[x], lane_v, k))};
        mma_f16_16816(O[i2], a, pb0, pb1);
      }
    } else if constexpr (VINTER) {
      // combine the two tokens of each pair word-wise: field c of lo/hi is
      // (code of token a) | (code of token b) << VB
      constexpr uint32_t M = VB == 1 ? 0x55555555u : VB == 2 ? 0x33333333u : 0x0F0F0F0Fu;
      uint32_t lab[VOW], hab[VOW], lcd[VOW], hcd[VOW];
#pragma unroll
      for (int x = 0; x < VOW; ++x) {
        lab[x] = (wa[x] & M) | ((wb[x] << VB) & ~M);
        hab[x] = ((wa[x] >> VB) & M) | (wb[x] & ~M);
        lcd[x] = (wc[x] & M) | ((wd[x] << VB) & ~M);
        hcd[x] = ((wc[x] >> VB) & M) | (wd[x] & ~M);
      }
      constexpr int PER = 32 / VB;                 // codes per word
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        const int c0 = 2 * i2;                     // even position -> lo, odd -> hi
        const int o = ((c0 % PER) & ~1) * VB + (c0 / PER) * 32;
        uint32_t a[4];
        a[0] = lds32(lutv, field_addr<2 * VB>(lab, o, lane4));
        a[1] = lds32(lutv, field_addr<2 * VB>(hab, o, lane4));
        a[2] = lds32(lutv, field_addr<2 * VB>(lcd, o, lane4));
        a[3] = lds32(lutv, field_addr<2 * VB>(hcd, o, lane4));
        mma_f16_16816(O[i2], a, pb0, pb1);
      }
    } else {
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        const int c0p = (2 * i2) * VB, c1p = (2 * i2 + 1) * VB;
        uint32_t a[4];
        if constexpr (Lut<VB>::kPair) {
          a[0] = lds32(lutv, (((getbits(wb, c0p, VB) << VB) | getbits(wa, c0p, VB)) << 7 | lane4));
          a[1] = lds32(lutv, (((getbits(wb, c1p, VB) << VB) | getbits(wa, c1p, VB)) << 7 | lane4));
          a[2] = lds32(lutv, (((getbits(wd, c0p, VB) << VB) | getbits(wc, c0p, VB)) << 7 | lane4));
          a[3] = lds32(lutv, (((getbits(wd, c1p, VB) << VB) | getbits(wc, c1p, VB)) << 7 | lane4));
        } else {
          a[0] = lds16(lutv, (getbits(wa, c0p, VB) << 1)) | (lds16(lutv, (getbits(wb, c0p, VB) << 1)) << 16);
          a[1] = lds16(lutv, (getbits(wa, c1p, VB) << 1)) | (lds16(lutv, (getbits(wb, c1p, VB) << 1)) << 16);
          a[2] = lds16(lutv, (getbits(wc, c0p, VB) << 1)) | (lds16(lutv, (getbits(wd, c0p, VB) << 1)) << 16);
          a[3] = lds16(lutv, (getbits(wc, c1p, VB) << 1)) | (lds16(lutv, (getbits(wd, c1p, VB) << 1)) << 16);
        }
        mma_f16_16816(O[i2], a, pb0, pb1);
      }
    }
  };

  // Segments are the runs of one stream's pages in the unit's range; the
  // group's warps take the segment's real pages in pairs, then combine their
  // partial results for the segment.
  const int cph = L.lens ? kSegPages : 0;       // placeholder pages opening a ragged stream
  int64_t s = s_first;                          // stream of the segment
  int64_t st0 = lay_start(L, s);                // its first compacted page
  int pg0 = (int)(gp0 - st0);                   // the segment's first page in the stream
  int i0 = 0;                                   // unit-relative index of that page
  int ring = 0;                                 // position in the group's stage ring
  uint32_t phase = 0;
  while (i0 < npages) {
    const int64_t st1 = lay_start(L, s + 1);
    const int i1 = (int)tmin<int64_t>(npages, i0 + (st1 - st0 - pg0));   // pages [i0, i1)
    const int Ts = lay_tokens(L, s);            // valid tokens of the stream
    const int Ks = lay_kstart(L, s);            // first attended token (left padding)
    const int ir0 = tmax(i0, i0 + cph - pg0);   // first real (non-placeholder) page
    if (ir0 < i1) load_q(s);
    for (int ip = ir0; ip < i1; ip += 2) {
      const int npair = tmin(2, i1 - ip);       // pages taken this round
      if (half < npair) {
        const int rp = ring + half;             // ring slot of this warp's page
        const int st = grp * G::SG + (rp >= G::SG ? rp - G::SG : rp);
        const uint32_t ph = phase ^ (rp >= G::SG ? 1u : 0u);
        if (!s_abort && !mbar_wait_poll(&full[st], ph)) {
          atomicOr(p.status, TQ_DEV_WAIT_TIMEOUT);
          s_abort = 1;
        }
        const uint8_t* pgb = stages + st * G::PB;
        const int pg = pg0 + (ip + half - i0) - cph;   // page in the stream (real)
        const int tokw = pg * kPageTokens + wt0;       // the warp's first token

        if (tokw < Ts && tokw + 32 > Ks) {
          float sc[2][4];
#pragma unroll
          for (int t = 0; t < 2; ++t) tile_scores(pgb, wt0 + 16 * t + gq, sc[t]);
          // rows beyond the stream's tokens or before its first attended
          // token take no weight (warp-uniform test: only a stream's first
          // and last pages hold such rows)
          const bool edge = tokw + 32 > Ts || tokw < Ks;
          if (edge) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int r = tokw + 16 * t + gq;
              if (r >= Ts || r < Ks) { sc[t][0] = kNegInf; sc[t][1] = kNegInf; }
              if (r + 8 >= Ts || r + 8 < Ks) { sc[t][2] = kNegInf; sc[t][3] = kNegInf; }
            }
          }
          // ---------------- online softmax over the 32 tokens (columns =
          // heads 2tq, 2tq+1).  The exponent bias is the running max m plus
          // kLazyBits: while no score exceeds it, p = exp2(s - bias) <= 1 and
          // the max needs no warp reduction; only then is m reduced across
          // the warp and O, l rescaled
          float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][2]), fmaxf(sc[1][0], sc[1][2]));
          float mx1 = fmaxf(fmaxf(sc[0][1], sc[0][3]), fmaxf(sc[1][1], sc[1][3]));
          if (__any_sync(0xffffffffu, mx0 > m0 + kLazyBits || mx1 > m1 + kLazyBits)) {
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
              mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
              mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            const float n0m = fmaxf(m0, mx0), n1m = fmaxf(m1, mx1);
            const float c0 = n0m == m0 ? 1.f : fast_exp2(m0 - n0m);
            const float c1 = n1m == m1 ? 1.f : fast_exp2(m1 - n1m);
            l0 *= c0;
            l1 *= c1;
#pragma unroll
            for (int i2 = 0; i2 < NJ; ++i2) {
              O[i2][0] *= c0; O[i2][2] *= c0;
              O[i2][1] *= c1; O[i2][3] *= c1;
            }
            m0 = n0m;
            m1 = n1m;
          }
          const float b0s = m0 == kNegInf ? 0.f : m0 + kLazyBits;
          const float b1s = m1 == kNegInf ? 0.f : m1 + kLazyBits;
          const __half* vn = reinterpret_cast<const __half*>(pgb + G::OFF_VN);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int r0 = wt0 + 16 * t + gq;
            const float p00 = fast_exp2(sc[t][0] - b0s), p01 = fast_exp2(sc[t][1] - b1s);
            const float p10 = fast_exp2(sc[t][2] - b0s), p11 = fast_exp2(sc[t][3] - b1s);
            l0 += p00 + p10;
            l1 += p01 + p11;
            // ---------------- P' = p * ||v|| -> B fragments ---------------
            // (a masked row has p = 0; its norm slot may be stale)
            const float v0 = __half2float(vn[r0]), v1 = __half2float(vn[r0 + 8]);
            uint32_t pb0, pb1;
            if (edge) {
              pb0 = movmatrix_trans(pack_half2(p00 == 0.f ? 0.f : p00 * v0, p01 == 0.f ? 0.f : p01 * v0));
              pb1 = movmatrix_trans(pack_half2(p10 == 0.f ? 0.f : p10 * v1, p11 == 0.f ? 0.f : p11 * v1));
            } else {
              pb0 = movmatrix_trans(pack_half2(p00 * v0, p01 * v0));
              pb1 = movmatrix_trans(pack_half2(p10 * v1, p11 * v1));
            }
            tile_pv(pgb, wt0 + 16 * t, pb0, pb1);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if constexpr (SELF) {
          // the pair's first warp refills the stage with the page SG later
          // once its partner has released it too (every page is real here, so
          // the unit-relative index is ip + half and the stage's use is r / SG)
          const int r = ip + half;
          if ((tw & 1) == 0 && lane == 0 && r + G::SG < npages && !s_abort) {
            if (mbar_wait_poll(&empty[st], (uint32_t)((r / G::SG) & 1))) {
              issue(st, gp0 + r + G::SG);
            } else {
              atomicOr(p.status, TQ_DEV_WAIT_TIMEOUT);
              s_abort = 1;
            }
          }
        }
      }
      ring += npair;
      if (ring >= G::SG) { ring -= G::SG; phase ^= 1u; }
    }

    // ---------------- segment end: combine warps, emit partial ---------------
    {
      float L0 = l0, L1 = l1;
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        L0 += __shfl_xor_sync(0xffffffffu, L0, o);
        L1 += __shfl_xor_sync(0xffffffffu, L1, o);
      }
      // the group is done with the K table (which the scratch aliases when
      // NG == 1), or with its previous segment's scratch
      group_bar<G::NG>(grp, GT);
      float* comb = reinterpret_cast<float*>(G::FAST ? smem + G::COMB_OFF : lutk);
      float* cm = comb + warp * (16 + 8 * D);
      float* cl = cm + 8;
      float* co = cm + 16;
      if (gq == 0) {                           // l and O are relative to m + kLazyBits
        cm[2 * tq] = m0 == kNegInf ? kNegInf : m0 + kLazyBits;
        cm[2 * tq + 1] = m1 == kNegInf ? kNegInf : m1 + kLazyBits;
        cl[2 * tq] = L0; cl[2 * tq + 1] = L1;
      }
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        co[(2 * tq) * D + 16 * i2 + gq] = O[i2][0];
        co[(2 * tq + 1) * D + 16 * i2 + gq] = O[i2][1];
        co[(2 * tq) * D + 16 * i2 + gq + 8] = O[i2][2];
        co[(2 * tq + 1) * D + 16 * i2 + gq + 8] = O[i2][3];
      }
      group_bar<G::NG>(grp, GT);
      const int64_t hrow0 = ((int64_t)hc * L.nid + unit + s) * 8;
      const float* gcomb = comb + grp * kTileWarps * (16 + 8 * D);
      for (int idx = gtid; idx < 8 * D; idx += GT) {
        const int h = idx / D, d = idx % D;
        float M = kNegInf;
#pragma unroll
        for (int w = 0; w < kTileWarps; ++w) M = fmaxf(M, gcomb[w * (16 + 8 * D) + h]);
        float Lsum = 0.f, Osum = 0.f;
        if (M != kNegInf) {
#pragma unroll
          for (int w = 0; w < kTileWarps; ++w) {
            const float* cw = gcomb + w * (16 + 8 * D);
            const float wt = fast_exp2(cw[h] - M);
            Lsum = fmaf(wt, cw[8 + h], Lsum);
            Osum = fmaf(wt, cw[16 + h * D + d], Osum);
          }
        }
        const int64_t hrow = hrow0 + h;
        p.part_o[hrow * D + d] = Osum;
        if (d == 0) {
          p.part_m[hrow] = M;
          p.part_l[hrow] = Lsum;
        }
      }
      if constexpr (!G::FAST) {                // NG == 1: the group is the CTA
        group_bar<G::NG>(grp, GT);
        if (i1 != npages) {                    // restore the table the scratch used
          build_lut<KB>(lutk, p.kc, gtid, GT);
          group_bar<G::NG>(grp, GT);
        }
      }
      reset_state();
    }
    i0 = i1;
    pg0 = 0;
    st0 = st1;
    ++s;
    // a ragged batch may hold empty streams: step to the next one with pages
    while (i0 < npages && lay_start(L, s + 1) == st0) ++s;
  }
  if constexpr (SELF) {
    // after a timed-out wait, never leave with a copy still writing shared
    // memory: the newest copy into each of the group's stages completes
    // after the older ones
    group_bar<G::NG>(grp, GT);
    if (s_abort && gtid < G::SG) {
      const int stg = grp * G::SG + gtid;
      const int n = s_issued[stg];
      if (n > 0) mbar_wait_bounded(&full[stg], (uint32_t)((n - 1) & 1), 16u);
    }
  }
}

// ---------------------------------------------------------------------------
// Query preparation (and, for a decode step, the append of the new token).
//
// q_rot = q R^T and Sq = S q_rot for the <= 8 query heads of a head chunk
// become fp16 fragments for decode_kernel (softmax scale * log2e folded in).
// With `append` set, the stream's new K/V token is stored at position `pos`,
// with the same math and summation order as append_kernel
// (kv_cache.py:382-398), so the page bytes are identical to a tq_append of
// that token: by the CTAs of head chunk 0 or, when the grid still fits one
// wave with it (`append_cta`: small batches), by one more CTA per stream
// (blockIdx.y == nch) that runs beside the query CTAs.  grid = (S, nch [+ 1]),
// 256 threads; thread (j, grp) owns output coordinate j of the vectors grp,
// grp + G, ... (G = 256 / D).
// ---------------------------------------------------------------------------
struct QPrepParams {
  int D, g, Hkv, nch;
  const void* q; int q_dtype; int64_t q_stride[4];
  const float* RT; const float* ST;   // R^T, S^T (row-major)
  float scale_q, scale_s;
  uint32_t* qf; uint32_t* sqf;
};

struct PrepParams {
  QPrepParams q;
  int append;
  PageGeom g;
  const float* kc; const float* kb; const float* vc; const float* vb;
  const void* kx; const void* vx; int k_dtype, v_dtype; int64_t ks[4], vs[4];
  uint8_t* pages; PageMap pm; int64_t pos;
  uint32_t* status;
  PageLayout lay;        // ragged (lay.lens set): store at row length - 1, lay out the pages
  int units;             // the decode's work units (CTAs x page groups)
  int append_cta;        // the append has its own CTA per stream (blockIdx.y == nch)
};

constexpr int kPrepThreads = 256;

// Ragged page layout, by all threads of one CTA: cum[s] = compacted pages of
// the streams before s, cum[S] = all pages, *rq = pages per unit (at least
// Pv / (kMaxSlots - 1), so no stream has more segments than the merge's slot
// table).  Each thread sums a run of rows; the run totals are scanned by warp
// shuffles.
constexpr int kMaxSlots = 64;

__device__ __noinline__ void ragged_layout(const PageLayout L, int units, int tid) {
  __shared__ int64_t s_warp[kPrepThreads / 32];
  const int lane = tid & 31, warp = tid >> 5;
  const int64_t B = L.S / L.hkv;
  const int64_t run = (B + kPrepThreads - 1) / kPrepThreads;
  const int64_t b0 = tmin<int64_t>(B, tid * run), b1 = tmin<int64_t>(B, b0 + run);
  auto row_pages = [&](int64_t b) {            // real pages + placeholders per stream
    const int64_t n = ((int64_t)lay_tokens(L, b * L.hkv) + kPageTokens - 1) / kPageTokens;
    return n > 0 ? n + kSegPages : 0;
  };
  int64_t mine = 0;
  for (int64_t b = b0; b < b1; ++b) mine += row_pages(b) * L.hkv;
  int64_t incl = mine;                            // inclusive scan within the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int64_t before = incl - mine, all = 0;
  for (int w = 0; w < kPrepThreads / 32; ++w) {
    if (w < warp) before += s_warp[w];
    all += s_warp[w];
  }
  for (int64_t b = b0; b < b1; ++b) {
    const int64_t pg = row_pages(b);
    for (int h = 0; h < L.hkv; ++h) L.cum[b * L.hkv + h] = (int32_t)(before + h * pg);
    before += pg * L.hkv;
  }
  if (tid == 0) {
    L.cum[L.S] = (int32_t)all;
    const int64_t q = tmax<int64_t>(tmax<int64_t>((all + units - 1) / tmax(units, 1), 1),
                                    (L.Pv + kSegPages + kMaxSlots - 2) / (kMaxSlots - 1));
    *L.rq = (int32_t)q;
  }
}

template <int D>
struct PrepSmem {
  // floats: R^T, S^T, xs[10][D] (q x8, k, v), ys[10][D], codebooks 4x256, norms 4;
  // then codes and order tables
  static size_t bytes(bool qjl) {
    return ((qjl ? 2 : 1) * (size_t)D * D + 20 * D + 4 * 256 + 4) * 4 + 3 * D + 3 * D * 2 + 16;
  }
};

template <int D, bool SEP>
__global__ void __launch_bounds__(kPrepThreads) prep_kernel(PrepParams pp) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int G = kPrepThreads / D;            // vector groups
  constexpr int NA = (10 + G - 1) / G;           // vectors per thread, phase A
  constexpr int NB = (9 + G - 1) / G;            // vectors per thread, phase B
  const QPrepParams& p = pp.q;
  const PageGeom& g = pp.g;
  const bool qjl = p.ST != nullptr;
  float* rt = reinterpret_cast<float*>(smem);    // [D][D] R^T
  float* stt = rt + D * D;                       // [D][D] S^T (QJL only)
  float* xs = stt + (qjl ? D * D : 0);           // [10][D]: q heads, u_k, u_v; later Sq
  float* ys = xs + 10 * D;                       // [10][D]: q_rot, y_k (-> residual), y_v
  float* cb = ys + 10 * D;                       // [4][256] k cent, k bnd, v cent, v bnd
  float* nrm = cb + 4 * 256;                     // ||k||, ||v||, gamma
  uint8_t* code = reinterpret_cast<uint8_t*>(nrm + 4);   // [2][D]
  uint8_t* qb = code + 2 * D;                    // [D]
  int16_t* ordk = reinterpret_cast<int16_t*>(qb + D);
  int16_t* ordv = ordk + D;
  int16_t* qinv = ordv + D;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int j = tid % D, grp = tid / D;
  const int64_t s = blockIdx.x;
  const int hc = blockIdx.y;
  const int64_t b = s / p.Hkv, kvh = s % p.Hkv;
  // SEP: the step's append has its own CTA (blockIdx.y == nch)
  const bool qrole = !SEP || hc < p.nch;         // query CTA (else the step's append CTA)
  const int nh = qrole ? tmin(8, p.g - hc * 8) : 0;
  const bool app = pp.append && (SEP ? !qrole : hc == 0);
  const int nbk = (1 << g.kb) - 1, nbv = (1 << g.vb) - 1;

  stage_async(rt, p.RT, D * D * 4, tid, kPrepThreads);
  if (qjl) stage_async(stt, p.ST, D * D * 4, tid, kPrepThreads);
  if (app) {
    // the layer's constant tables: read before the dependency wait, so their
    // latency overlaps the previous kernel
    for (int i = tid; i < 256; i += kPrepThreads) {
      if (i <= nbk) cb[i] = pp.kc[i];
      if (i < nbk) cb[256 + i] = pp.kb[i];
      if (i <= nbv) cb[512 + i] = pp.vc[i];
      if (i < nbv) cb[768 + i] = pp.vb[i];
    }
    build_orders(ordk, ordv, qinv, D, tid, kPrepThreads);
  }
  pdl_launch_dependents();
  pdl_wait();
  if (qrole) {
    for (int i = tid; i < 8 * D; i += kPrepThreads) {
      const int hl = i / D, c = i % D;
      xs[i] = hl < nh ? load_elem(p.q, p.q_dtype, b * p.q_stride[0] +
                                  (kvh * p.g + hc * 8 + hl) * p.q_stride[1] + c * p.q_stride[3])
                      : 0.f;
      if (hl >= nh) ys[i] = 0.f;                 // padded heads: zero fragments, not computed
    }
  }
  if (app) {
    if (warp == 0) {
      const float n = warp_normalize(pp.kx, pp.k_dtype, b * pp.ks[0] + kvh * pp.ks[1], pp.ks[3],
                                     xs + 8 * D, D, lane);
      if (lane == 0) nrm[0] = n;
    } else if (warp == 1) {
      const float n = warp_normalize(pp.vx, pp.v_dtype, b * pp.vs[0] + kvh * pp.vs[1], pp.vs[3],
                                     xs + 9 * D, D, lane);
      if (lane == 0) nrm[1] = n;
    }
  }
  cp_async_wait_all();
  __syncthreads();

  // phase A: rotate the nh real query heads (and u_k, u_v); vector a of the
  // active list sits at row a (a head) or 8 + a - nh (u_k, u_v).  The loop
  // is bound by shared-memory wavefronts, one per (vector, i) and warp, so
  // the heads a GQA group pads to 8 are not computed.  (A tensor-core
  // rotation of the heads with bf16 terms of R, B fragments read from L2,
  // measured slower: 14.8 against 10.7 us per call.)
  {
    const int nvec = nh + (app ? 2 : 0);
    const int mine = (grp < G && nvec > grp) ? (nvec - grp + G - 1) / G : 0;
    const int nhl = nh;
    int row[NA];
#pragma unroll
    for (int k = 0; k < NA; ++k) {
      const int a = grp + k * G;
      row[k] = a < nhl ? a : tmin(8 + a - nhl, 9);
    }
    float acc[NA];
    rot_rows<D, NA>(xs, row, mine, rt, j, acc);
#pragma unroll
    for (int k = 0; k < NA; ++k) {
      const int v = row[k];
      if (k < mine) {
        ys[v * D + j] = acc[k];
        if (v == 8) code[j] = (uint8_t)bucketize_lt(cb + 256, nbk, acc[k]);
        if (v == 9) code[D + j] = (uint8_t)bucketize_lt(cb + 768, nbv, acc[k]);
      }
    }
  }
  __syncthreads();
  if (qjl) {
    if (app && tid < D) ys[8 * D + tid] -= cb[code[tid]];   // K residual y - c[idx]
    __syncthreads();
    // phase B: S q_rot for the nh heads, S r for the K residual (row 8)
    const int nhl = nh;
    const int nvec = nhl + (app ? 1 : 0);
    const int mine = (grp < G && nvec > grp) ? (nvec - grp + G - 1) / G : 0;
    int row[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int a = grp + k * G;
      row[k] = a < nhl ? a : 8;
    }
    float acc[NB];
    rot_rows<D, NB>(ys, row, mine, stt, j, acc);
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int v = row[k];
      if (k < mine) {
        if (v < 8) xs[v * D + j] = acc[k];
        else qb[j] = acc[k] >= 0.f ? 1 : 0;
      }
    }
    if (app && warp == 0) {
      float ss = 0.f;
      for (int c = lane; c < D; c += 32) ss = fmaf(ys[8 * D + c], ys[8 * D + c], ss);
      ss = warp_sum(ss);
      if (lane == 0) nrm[2] = nrm[0] * sqrtf(ss);
    }
  }
  __syncthreads();
  if (qrole) {
    uint32_t* qo = p.qf + (s * p.nch + hc) * 8 * (D / 2);
    for (int i = tid; i < 8 * (D / 2); i += kPrepThreads) {
      const int hl = i / (D / 2), c2 = i % (D / 2);
      qo[i] = pack_half2(ys[hl * D + 2 * c2] * p.scale_q, ys[hl * D + 2 * c2 + 1] * p.scale_q);
    }
  }
  if (qjl && qrole) {
    uint32_t* so = p.sqf + (s * p.nch + hc) * 8 * (D / 2);
    for (int i = tid; i < 8 * (D / 2); i += kPrepThreads) {
      const int hl = i / (D / 2), c2 = i % (D / 2);
      so[i] = pack_half2(xs[hl * D + 2 * c2] * p.scale_s, xs[hl * D + 2 * c2 + 1] * p.scale_s);
    }
  }
  bool page_ok = true;
  int64_t pslot = 0;
  // a ragged row stores its token at its length - 1 (not at all when empty)
  const int64_t t = pp.lay.lens ? (int64_t)lay_tokens(pp.lay, s) - 1 : pp.pos;
  if (app && t >= 0) {
    pslot = page_slot(pp.pm, s, t / kPageTokens, page_ok);
    if (!page_ok && tid == 0) atomicOr(pp.status, TQ_DEV_BAD_BLOCK);
  }
  if (app && t >= 0 && page_ok) {
    uint8_t* page = pp.pages + pslot * (int64_t)g.page_bytes;
    const int slot = (int)(t % kPageTokens);
    const int kw = g.krow / 4, vw = g.vrow / 4, qw = qjl ? D / 32 : 0;
    // every word of the token's K, V and QJL rows is one warp ballot (lane b
    // holds bit b; the bit order of pack_word and pack_qjl_word), the words
    // spread over the CTA's warps
    for (int i = warp; i < kw + vw + qw; i += kPrepThreads / 32) {
      uint32_t word;
      uint32_t* dst;
      if (i < kw) {
        word = ballot_word(code, ordk, g.kb, i, D, lane);
        dst = reinterpret_cast<uint32_t*>(page + g.off_k + slot * g.krow) + i;
      } else if (i < kw + vw) {
        word = ballot_word(code + D, ordv, g.vb, i - kw, D, lane);
        dst = reinterpret_cast<uint32_t*>(page + g.off_v + slot * g.vrow) + (i - kw);
      } else {
        word = __ballot_sync(0xffffffffu, qb[qinv[32 * (i - kw - vw) + lane]] != 0);
        dst = reinterpret_cast<uint32_t*>(page + g.off_q + slot * g.qrow) + (i - kw - vw);
      }
      if (lane == 0) *dst = word;
    }
    if (tid == 0) {
      reinterpret_cast<__half*>(page + g.off_kn)[slot] = __float2half_rn(nrm[0]);
      reinterpret_cast<__half*>(page + g.off_vn)[slot] = __float2half_rn(nrm[1]);
      if (qjl) reinterpret_cast<__half*>(page + g.off_kr)[slot] = __float2half_rn(nrm[2]);
    }
  }
  if (pp.lay.lens && blockIdx.x == 0 && blockIdx.y == 0) ragged_layout(pp.lay, pp.units, tid);
}

// ---------------------------------------------------------------------------
// merge: combine partials, add the window, un-rotate, store
// grid = (S, nch), 128 threads
// ---------------------------------------------------------------------------
struct MergeParams {
  int D, g, Hkv, nch;
  PageLayout lay;
  const float* part_m; const float* part_l; const float* part_o;
  const float* R;
  const void* q; int q_dtype; int64_t q_stride[4];
  const void* wk; const void* wv; int w_dtype; int64_t wk_stride[4], wv_stride[4]; int64_t W;
  float scale_log2;       // softmax scale * log2(e)
  void* out; int out_dtype; int64_t out_stride[4];
  // fused output all-gather (world > 1): the block goes to every rank's
  // buffer, then each CTA adds 1 to every rank's arrival counter
  int world, rank;
  void* peer_out[TQ_MAX_PEERS];
  uint32_t* peer_flag[TQ_MAX_PEERS];   // [arrivals, this rank's finished CTAs]
  uint32_t* status;
  int hpc;                // heads per CTA: CTA z of (stream, chunk) takes heads [z hpc, (z + 1) hpc)
};

constexpr int kMergeThreads = 256;
constexpr int kSlotChunk = 8;

// grid = (S, nch, ceil(heads / hpc)), 256 threads: with few streams the
// heads of a chunk are spread over CTAs, so each stages and combines only
// its own heads' partials (a long-context batch of 8 streams has ~50 slots
// per stream).  Shared memory: R [D][D], the rotated combination orot
// [8][D], a chunk of partials [slots][heads][D] (8 * kSlotChunk * D floats),
// and for the window q [8][D] and scores/probabilities [8][W].
template <int D, bool SPLIT>
__global__ void __launch_bounds__(kMergeThreads) merge_kernel(MergeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int64_t W = p.W;
  float* rs = reinterpret_cast<float*>(smem);     // [D][D] R
  float* orot = rs + D * D;                        // [8][D]
  float* po = orot + 8 * D;                        // [8][kSlotChunk][D]
  float* qv = po + 8 * kSlotChunk * D;             // [8][D]  (window only)
  float* sc = qv + 8 * D;                          // [8][W]  (window only)
  __shared__ float s_wt[8][kMaxSlots];
  __shared__ float s_M[8], s_L[8];
  const int64_t s = blockIdx.x;
  const int hc = blockIdx.y;
  const int64_t b = s / p.Hkv, kvh = s % p.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NWARP = kMergeThreads / 32;
  const int nh = tmin(8, p.g - hc * 8);
  // SPLIT: this CTA's heads are [ha, hb) of the chunk and it stages only
  // their rows; otherwise it takes the whole chunk and stages all 8 head rows
  // of a slot (one contiguous run per chunk of slots)
  constexpr bool whole = !SPLIT;
  const int ha = SPLIT ? (int)blockIdx.z * p.hpc : 0;
  const int hb = SPLIT ? tmin(nh, ha + p.hpc) : nh;
  const int hn = tmax(0, hb - ha);
  const int kcap = whole ? kSlotChunk : (8 * kSlotChunk) / tmax(hn, 1);   // slots per chunk
  stage_async(rs, p.R, D * D * 4, tid, kMergeThreads);
  pdl_launch_dependents();
  pdl_wait();
  // the stream's segments: CTAs first .. last of the decode, ids first + s ..
  int nslot = 0;
  int64_t hrow0 = 0;                               // (chunk, id) row of the first segment, x 8
  {
    const PageLayout& L = p.lay;
    const int64_t Q = L.lens ? (int64_t)__ldcg(L.rq) : L.Q;
    const int64_t a0 = lay_start(L, s), a1 = lay_start(L, s + 1);
    if (a1 > a0) {
      const int64_t first = a0 / Q;
      // <= kMaxSlots: Q >= Pv / (kMaxSlots - 1) on both layouts (the clamp
      // only keeps the slot table in bounds)
      nslot = tmin((int)((a1 - 1) / Q - first + 1), kMaxSlots);
      hrow0 = ((int64_t)hc * L.nid + first + s) * 8;
    }
  }
  // slots k0 .. k0 + kn - 1 of heads [ha, hb) into po[k - k0][h - ha][D]
  auto stage_chunk = [&](int k0, int kn) {
    if constexpr (whole) {                         // one run: rows are (slot, head)
      stage_async(po, p.part_o + (hrow0 + 8 * k0) * D, kn * 8 * D * 4, tid, kMergeThreads);
    } else {
      for (int k = 0; k < kn; ++k)
        stage_async(po + k * hn * D, p.part_o + (hrow0 + 8 * (k0 + k) + ha) * D, hn * D * 4, tid,
                    kMergeThreads);
    }
  };
  // the first chunk of partials starts copying now, behind the window and
  // per-head passes
  if (nslot > 0 && hn > 0) stage_chunk(0, tmin(kcap, nslot));

  // --- window scores (unrotated), all heads --------------------------------
  if (W > 0) {
    for (int i = tid; i < 8 * D; i += kMergeThreads) {
      const int hl = i / D, c = i % D;
      qv[i] = (hl >= ha && hl < hb) ? load_elem(p.q, p.q_dtype, b * p.q_stride[0] +
                                  (kvh * p.g + hc * 8 + hl) * p.q_stride[1] + c * p.q_stride[3])
                      : 0.f;
    }
    __syncthreads();
    for (int64_t t = warp; t < W; t += NWARP) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int c = lane; c < D; c += 32) {
        const float kx = load_elem(p.wk, p.w_dtype, b * p.wk_stride[0] + kvh * p.wk_stride[1] +
                                                        t * p.wk_stride[2] + c * p.wk_stride[3]);
#pragma unroll
        for (int h = 0; h < 8; ++h) acc[h] = fmaf(qv[h * D + c], kx, acc[h]);
      }
      // window token t sits at position (the row's packed tokens) + t
      const bool masked = lay_tokens(p.lay, s) + t < lay_kstart(p.lay, s);
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        const float v = warp_sum(acc[h]);
        if (lane == 0) sc[h * W + t] = masked ? kNegInf : v * p.scale_log2;
      }
    }
    __syncthreads();
  }
  // --- per-head max and partial weights: warp h handles head h ---------------
  if (warp < 8) {
    const int h = warp;
    float M = kNegInf;
    // slots lane and lane + 32 (kMaxSlots = 64): m and l loaded together
    static_assert(kMaxSlots <= 64, "two slots per lane");
    float mk[2] = {kNegInf, kNegInf}, lk[2] = {0.f, 0.f};
    const bool mine = h >= ha && h < hb;
    if (mine) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int k = lane + 32 * u;
        if (k < nslot) {
          mk[u] = p.part_m[hrow0 + 8 * k + h];
          lk[u] = p.part_l[hrow0 + 8 * k + h];
        }
      }
      M = fmaxf(mk[0], mk[1]);
      for (int64_t t = lane; t < W; t += 32) M = fmaxf(M, sc[h * W + t]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float Ms = M == kNegInf ? 0.f : M;
    float L = 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int k = lane + 32 * u;
      if (k < nslot) {
        const float wt = (mine && mk[u] != kNegInf) ? exp2f(mk[u] - Ms) : 0.f;
        s_wt[h][k] = wt;
        L = fmaf(wt, lk[u], L);
      }
    }
    for (int64_t t = lane; t < W; t += 32) {
      const float e = mine ? exp2f(sc[h * W + t] - Ms) : 0.f;
      sc[h * W + t] = e;
      L += e;
    }
    L = warp_sum(L);
    if (lane == 0) { s_M[h] = Ms; s_L[h] = L; }
  }
  __syncthreads();
  // --- rotated partial combination, slots staged in chunks ------------------
  constexpr int OUT = 4;                          // outputs per thread (8 * 128 / 256)
  float acc[OUT] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; hn > 0 && k0 < nslot; k0 += kcap) {
    const int kn = tmin(kcap, nslot - k0);
    // (the first chunk was issued after the dependency wait)
    if (k0 > 0) stage_chunk(k0, kn);
    cp_async_wait_all();
    __syncthreads();
    if constexpr (whole) {
#pragma unroll
      for (int r = 0; r < OUT; ++r) {
        const int i = tid + r * kMergeThreads;
        if (i < 8 * D) {
          const int h = i / D, d = i % D;
          for (int k = 0; k < kn; ++k) acc[r] = fmaf(s_wt[h][k0 + k], po[(k * 8 + h) * D + d], acc[r]);
        }
      }
    } else {
#pragma unroll
      for (int r = 0; r < OUT; ++r) {
        const int i = tid + r * kMergeThreads;
        if (i < hn * D) {
          const int hl = i / D, d = i % D;
          for (int k = 0; k < kn; ++k)
            acc[r] = fmaf(s_wt[ha + hl][k0 + k], po[(k * hn + hl) * D + d], acc[r]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < OUT; ++r) {
    const int i = tid + r * kMergeThreads;
    if (whole ? i < 8 * D : i < hn * D) orot[(whole ? 0 : ha * D) + i] = acc[r];
  }
  cp_async_wait_all();
  __syncthreads();
  // --- un-rotate (o = O_rot R), add the window, normalise, store --------------
  // thread (j, grp) handles heads grp*hpg .. grp*hpg + hpg-1 of coordinate
  // j.  A group of at most hpg heads (GQA 4 at D128) would leave the other
  // thread groups idle, so there every group sums its own part of the
  // d-range for heads 0 .. hpg-1 and group 0 adds the parts, in order,
  // through the partial buffer (consumed by now).
  constexpr int groups = kMergeThreads / D;       // 2 for D = 128
  constexpr int hpg = 8 / groups;                 // heads per group
  static_assert(D * groups == kMergeThreads && groups * hpg * D <= 8 * kSlotChunk * D, "merge");
  const bool split = groups > 1 && hn <= hpg;     // block-uniform
  const int j = tid % D, grp = tid / D;
  // rows h0 + h beyond 7 (a CTA's last heads) read row 7 and are never stored
  const int h0 = split ? ha : ha + grp * hpg;
  const int d0 = split ? grp * (D / groups) : 0, d1 = split ? d0 + D / groups : D;
  float o[hpg];
#pragma unroll
  for (int h = 0; h < hpg; ++h) o[h] = 0.f;
  if (h0 < hb) {
#pragma unroll 4
    for (int d = d0; d < d1; ++d) {
      const float r = rs[d * D + j];
#pragma unroll
      for (int h = 0; h < hpg; ++h) o[h] = fmaf(orot[tmin(h0 + h, 7) * D + d], r, o[h]);
    }
  }
  if (split) {
#pragma unroll
    for (int h = 0; h < hpg; ++h) po[(grp * hpg + h) * D + j] = o[h];
    __syncthreads();
    if (grp == 0)
      for (int q = 1; q < groups; ++q)
#pragma unroll
        for (int h = 0; h < hpg; ++h) o[h] += po[(q * hpg + h) * D + j];
  }
  if (split ? grp == 0 : h0 < hb) {
    for (int64_t t = 0; t < W; ++t) {
      const float vx = load_elem(p.wv, p.w_dtype, b * p.wv_stride[0] + kvh * p.wv_stride[1] +
                                                      t * p.wv_stride[2] + j * p.wv_stride[3]);
#pragma unroll
      for (int h = 0; h < hpg; ++h) o[h] = fmaf(sc[tmin(h0 + h, 7) * W + t], vx, o[h]);
    }
#pragma unroll
    for (int h = 0; h < hpg; ++h) {
      const int hh = h0 + h;
      if (hh >= hb) break;
      const float L = s_L[hh];
      const int64_t hq = kvh * p.g + hc * 8 + hh;
      const int64_t off = b * p.out_stride[0] + hq * p.out_stride[1] + j * p.out_stride[3];
      const float v = L > 0.f ? o[h] / L : 0.f;
      if (p.world <= 1) {
        store_elem(p.out, p.out_dtype, off, v);
      } else {
        for (int r = 0; r < p.world; ++r) store_elem(p.peer_out[r], p.out_dtype, off, v);
      }
    }
  }
  if (p.world > 1) {
    // Completion of the fused all-gather.  The CTA's barrier orders all its
    // threads' peer stores before thread 0, which counts the CTA done on its
    // own GPU with a release at GPU scope.  The rank's last CTA acquires the
    // other CTAs' counts, so every store of the rank precedes it in causality
    // order; one system-scope fence then orders them all before the plain
    // arrivals it adds to every rank's counter (fence + relaxed add = one
    // release per peer), and it waits until its own counter reaches
    // (calls completed + 1) * world.  One system fence per rank and call
    // instead of one per CTA plus a release per peer: measured at 2 GPUs the
    // per-CTA fences took 3.7 us and the per-peer releases 4.6 us of every
    // layer.  The counter only grows (wrap-safe compare), so a late arrival
    // after a timed-out wait still lands in its own call's count, and no rank
    // can arrive twice before every rank has arrived once (its next arrival
    // needs its own wait to have passed).
    __syncthreads();
    if (tid == 0) {
      uint32_t* arrived = p.peer_flag[p.rank];
      uint32_t* done = arrived + 1;
      uint32_t* calls = arrived + 2;
      const uint32_t nctas = gridDim.x * gridDim.y * gridDim.z;
      uint32_t prev;
      asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(done)
                   : "memory");
      if (prev + 1u == nctas) {
        // every other CTA of this rank has finished: acquire their counts,
        // and reset the local count for the layer's next call (which starts
        // after this grid completes)
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        *done = 0u;
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < p.world; ++r)
          asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p.peer_flag[r]) : "memory");
        const uint32_t ncall = *calls + 1u;
        const uint32_t target = ncall * (uint32_t)p.world;
        uint64_t t0 = 0;
        for (uint32_t i = 0;; ++i) {
          uint32_t v;
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(arrived) : "memory");
          if ((int32_t)(v - target) >= 0) break;
          if ((i & 255u) == 255u) {
            const uint64_t t = global_ns();
            if (t0 == 0) t0 = t;
            else if (t - t0 > 2000000000ull) { atomicOr(p.status, TQ_DEV_WAIT_TIMEOUT); break; }
          }
        }
        *calls = ncall;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

// Workspace: [0, 4) the status word, [64, 68) a ragged batch's pages per
// work unit, then the query fragments, the partials and a ragged page layout.
constexpr size_t kWsRaggedQ = 64;

struct Plan {
  int D, g, nch, ctas, units;
  int64_t S, Pv, T, Q, nid;
  size_t off_qf, off_sqf, off_m, off_l, off_o, off_cum, total;
};

using DecodeFn = void (*)(DecodeParams);

template <int D, int KB, int VB, bool QJL>
size_t dec_smem_bytes() { return (size_t)Dec<D, KB, VB, QJL>::SMEM; }

struct Variant {
  int D, kb, vb, qjl;
  DecodeFn fn;
  size_t (*smem)();
  int threads;
  int ng;                 // page groups (work units) per CTA
};

#define TQ_VARIANT(D_, KB_, VB_, Q_) \
  {D_, KB_, VB_, Q_, decode_kernel<D_, KB_, VB_, (Q_ != 0)>, dec_smem_bytes<D_, KB_, VB_, (Q_ != 0)>, \
   Dec<D_, KB_, VB_, (Q_ != 0)>::THREADS, Dec<D_, KB_, VB_, (Q_ != 0)>::NG}
#define TQ_VARIANT2(D_, KB_, VB_) TQ_VARIANT(D_, KB_, VB_, 0), TQ_VARIANT(D_, KB_, VB_, 1)

const Variant kVariants[] = {
    TQ_VARIANT2(128, 4, 2), TQ_VARIANT2(128, 3, 3), TQ_VARIANT2(128, 2, 2),
    TQ_VARIANT2(128, 4, 4), TQ_VARIANT2(128, 6, 4), TQ_VARIANT2(128, 5, 5),
    TQ_VARIANT2(128, 6, 6), TQ_VARIANT2(128, 8, 8),
    TQ_VARIANT2(64, 3, 3),  TQ_VARIANT2(64, 4, 2),  TQ_VARIANT2(64, 6, 4),
    TQ_VARIANT2(64, 5, 5),  TQ_VARIANT2(64, 4, 4),  TQ_VARIANT2(64, 2, 2),
    TQ_VARIANT2(32, 4, 2),  TQ_VARIANT2(32, 6, 4),  TQ_VARIANT2(32, 3, 3),
    TQ_VARIANT2(32, 5, 5),
};

// The self-fed kernels of the FAST variants (uniform batches on contiguous
// pages): same shared memory and work units, no producer warp.
struct SelfVariant {
  int vb, qjl;
  DecodeFn fn;
  int threads;
};
#define TQ_SELF_VARIANT(VB_, Q_) \
  {VB_, Q_, decode_kernel<128, 4, VB_, (Q_ != 0), true>, 32 * Dec<128, 4, VB_, (Q_ != 0)>::NCW}
const SelfVariant kSelfVariants[] = {
    TQ_SELF_VARIANT(2, 0), TQ_SELF_VARIANT(2, 1), TQ_SELF_VARIANT(4, 0), TQ_SELF_VARIANT(4, 1),
};

const SelfVariant* find_self_variant(const tq_geom* g, const tq_cache* c,
                                     const tq_decode_args* a) {
  if (g->head_dim != 128 || g->key_bits != 4 || a->seq_lens || c->block_table) return nullptr;
  for (const SelfVariant& v : kSelfVariants)
    if (v.vb == g->value_bits && v.qjl == (g->qjl != 0)) return &v;
  return nullptr;
}

const Variant* find_variant(const tq_geom* g) {
  for (const Variant& v : kVariants)
    if (v.D == g->head_dim && v.kb == g->key_bits && v.vb == g->value_bits && v.qjl == (g->qjl != 0))
      return &v;
  return nullptr;
}

Plan make_plan(const tq_geom* G, const tq_cache* c, const tq_decode_args* a, int occ, int ng) {
  Plan pl;
  pl.D = G->head_dim;
  const int64_t Hkv = c->streams / a->q->shape[0];
  pl.g = (int)(a->num_q_heads / Hkv);
  pl.nch = (pl.g + 7) / 8;
  pl.S = c->streams;
  pl.T = a->n_tokens;
  pl.Pv = (pl.T + kPageTokens - 1) / kPageTokens;
  const int64_t TP = pl.S * pl.Pv;
  int64_t slots = a->num_ctas > 0 ? a->num_ctas : (int64_t)device_sm_count() * tmax(occ, 1);
  slots = tmax<int64_t>(1, slots / tmax(pl.nch, 1));
  const int64_t want = slots * ng;               // work units: CTAs x page groups
  pl.Q = TP > 0 ? (TP + want - 1) / want : 1;    // pages per unit
  // every stream's partials must fit the merge kernel's slot table
  if (pl.Pv > 0) pl.Q = tmax<int64_t>(pl.Q, (pl.Pv + kMaxSlots - 2) / (kMaxSlots - 1));
  const int64_t used = TP > 0 ? (TP + pl.Q - 1) / pl.Q : 0;
  pl.ctas = (int)((used + ng - 1) / ng);
  pl.units = pl.ctas * ng;
  // a ragged batch has at most TP pages, so it keeps this grid and takes
  // fewer pages per unit; its segment ids stay below units + S as well
  pl.nid = pl.units + pl.S;
  size_t off = 256;
  const size_t heads = (size_t)pl.S * pl.nch * 8;
  const size_t rows = (size_t)pl.nch * pl.nid * 8;
  pl.off_qf = off;  off += heads * (pl.D / 2) * 4;
  pl.off_sqf = off; off += heads * (pl.D / 2) * 4;
  off = (off + 255) & ~(size_t)255;
  pl.off_m = off;   off += rows * 4;
  pl.off_l = off;   off += rows * 4;
  off = (off + 255) & ~(size_t)255;
  pl.off_o = off;   off += rows * pl.D * 4;
  pl.off_cum = off; off += ((size_t)pl.S + 1) * 4;
  pl.total = (off + 255) & ~(size_t)255;
  return pl;
}

int occupancy_of(const Variant* v, size_t smem) {
  return occupancy((const void*)v->fn, v->threads, smem);
}

}  // namespace

size_t decode_workspace_bytes(const tq_geom* g, const tq_cache* c, const tq_decode_args* a) {
  const Variant* v = find_variant(g);
  if (!v) return 0;
  const size_t smem = v->smem();
  if (set_smem_attr((const void*)v->fn, smem) != TQ_OK) return 0;
  return make_plan(g, c, a, occupancy_of(v, smem), v->ng).total;
}

using PrepFn = void (*)(PrepParams);

static bool prep_for(int D, PrepFn* fn, size_t* smem, bool qjl, bool sep) {
  switch (D) {
    case 32: *fn = sep ? prep_kernel<32, true> : prep_kernel<32, false>;
      *smem = PrepSmem<32>::bytes(qjl); return true;
    case 64: *fn = sep ? prep_kernel<64, true> : prep_kernel<64, false>;
      *smem = PrepSmem<64>::bytes(qjl); return true;
    case 128: *fn = sep ? prep_kernel<128, true> : prep_kernel<128, false>;
      *smem = PrepSmem<128>::bytes(qjl); return true;
    default: return false;
  }
}

int launch_decode(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                  const tq_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t st,
                  const StepInput* step) {
  const Variant* v = find_variant(G);
  if (!v) {
    set_error("tq_decode_attn: no kernel for head_dim=%d key_bits=%d value_bits=%d qjl=%d",
              G->head_dim, G->key_bits, G->value_bits, G->qjl);
    return TQ_ERR_INVALID;
  }
  const size_t smem = v->smem();
  if (set_smem_attr((const void*)v->fn, smem) != TQ_OK) return TQ_ERR_CUDA;
  const Plan pl = make_plan(G, c, a, occupancy_of(v, smem), v->ng);
  if (ws == nullptr || ws_bytes < pl.total) {
    set_error("tq_decode_attn: workspace of %zu bytes needed, %zu given", pl.total, ws_bytes);
    return TQ_ERR_WORKSPACE;
  }
  uint8_t* w = static_cast<uint8_t*>(ws);
  const int64_t Hkv = c->streams / a->q->shape[0];
  const float alpha = sqrtf(3.14159265358979f / 2.f) / (float)pl.D;
  const int phases = a->phases ? a->phases : (TQ_PHASE_QPREP | TQ_PHASE_DECODE | TQ_PHASE_MERGE);
  if (a->seq_lens && pl.S * (pl.Pv + kSegPages) >= ((int64_t)1 << 31)) {
    set_error("tq_decode_attn: a ragged batch needs streams x (pages + %d) < 2^31", kSegPages);
    return TQ_ERR_INVALID;
  }
  PageLayout lay;
  lay.S = pl.S; lay.Pv = pl.Pv; lay.T = pl.T; lay.Q = pl.Q;
  lay.hkv = (int)Hkv; lay.nid = pl.nid;
  lay.lens = a->seq_lens;
  lay.kstart = a->kv_start;
  lay.cum = reinterpret_cast<int32_t*>(w + pl.off_cum);
  lay.rq = reinterpret_cast<int32_t*>(w + kWsRaggedQ);

  QPrepParams qp;
  qp.D = pl.D; qp.g = pl.g; qp.Hkv = (int)Hkv; qp.nch = pl.nch;
  qp.q = a->q->data; qp.q_dtype = a->q->dtype;
  for (int i = 0; i < 4; ++i) qp.q_stride[i] = a->q->stride[i];
  qp.RT = t->rot_t; qp.ST = G->qjl ? t->qjl_t : nullptr;
  qp.scale_q = a->scale * kLog2e;
  qp.scale_s = a->scale * kLog2e * alpha;
  qp.qf = reinterpret_cast<uint32_t*>(w + pl.off_qf);
  qp.sqf = reinterpret_cast<uint32_t*>(w + pl.off_sqf);
  if (pl.S > 0 && (step || (phases & TQ_PHASE_QPREP))) {
    PrepParams pp;
    pp.lay = lay;
    pp.units = pl.units;
    pp.q = qp;
    pp.append = step != nullptr;
    pp.g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
    pp.kc = t->k_centroids; pp.kb = t->k_boundaries;
    pp.vc = t->v_centroids; pp.vb = t->v_boundaries;
    pp.kx = pp.vx = nullptr; pp.k_dtype = pp.v_dtype = 0;
    for (int i = 0; i < 4; ++i) pp.ks[i] = pp.vs[i] = 0;
    pp.pages = c->pages; pp.pm = page_map(c); pp.pos = 0;
    pp.status = reinterpret_cast<uint32_t*>(ws);
    if (step) {
      pp.kx = step->k->data; pp.vx = step->v->data;
      pp.k_dtype = step->k->dtype; pp.v_dtype = step->v->dtype;
      for (int i = 0; i < 4; ++i) { pp.ks[i] = step->k->stride[i]; pp.vs[i] = step->v->stride[i]; }
      pp.pos = step->pos;
    }
    PrepFn pfn;
    size_t psmem;
    // the step's append gets its own CTA per stream where the grid stays
    // within one wave (prep CTAs take most of an SM's shared memory)
    pp.append_cta = step && pl.S * (pl.nch + 1) <= (int64_t)device_sm_count();
    if (!prep_for(pl.D, &pfn, &psmem, G->qjl != 0, pp.append_cta != 0)) {
      set_error("tq_decode_attn: head_dim %d has no query-preparation kernel", pl.D);
      return TQ_ERR_INVALID;
    }
    if (set_smem_attr((const void*)pfn, psmem) != TQ_OK) return TQ_ERR_CUDA;
    const unsigned prep_y = (unsigned)(pl.nch + (pp.append_cta ? 1 : 0));
    if (launch_result(launch_pdl(pfn, dim3((unsigned)pl.S, prep_y), dim3(kPrepThreads), psmem, st, pp),
                      step ? "tq_decode_step/prep" : "tq_decode_attn/qprep") != TQ_OK)
      return TQ_ERR_CUDA;
  }

  DecodeParams dp;
  dp.pages = c->pages; dp.pm = page_map(c);
  dp.lay = lay;
  dp.nch = pl.nch;
  dp.qf = qp.qf; dp.sqf = qp.sqf;
  dp.kc = t->k_centroids; dp.vc = t->v_centroids;
  dp.part_m = reinterpret_cast<float*>(w + pl.off_m);
  dp.part_l = reinterpret_cast<float*>(w + pl.off_l);
  dp.part_o = reinterpret_cast<float*>(w + pl.off_o);
  dp.status = reinterpret_cast<uint32_t*>(w);
  if (pl.ctas > 0 && (phases & TQ_PHASE_DECODE)) {
    DecodeFn dfn = v->fn;
    int dthreads = v->threads;
    if (const SelfVariant* sv = find_self_variant(G, c, a)) {
      if (set_smem_attr((const void*)sv->fn, smem) != TQ_OK) return TQ_ERR_CUDA;
      dfn = sv->fn;
      dthreads = sv->threads;
    }
    if (launch_result(launch_pdl(dfn, dim3(pl.ctas, pl.nch), dim3(dthreads), smem, st, dp),
                      "tq_decode_attn/decode") != TQ_OK)
      return TQ_ERR_CUDA;
  }

  MergeParams mp;
  mp.D = pl.D; mp.g = pl.g; mp.Hkv = (int)Hkv; mp.nch = pl.nch;
  mp.lay = lay;
  mp.part_m = dp.part_m; mp.part_l = dp.part_l; mp.part_o = dp.part_o;
  mp.R = t->rot;
  mp.q = a->q->data; mp.q_dtype = a->q->dtype;
  for (int i = 0; i < 4; ++i) mp.q_stride[i] = a->q->stride[i];
  mp.W = 0; mp.wk = mp.wv = nullptr; mp.w_dtype = 0;
  for (int i = 0; i < 4; ++i) mp.wk_stride[i] = mp.wv_stride[i] = 0;
  if (a->window_k && a->window_v && a->window_k->shape[2] > 0) {
    mp.W = a->window_k->shape[2];
    mp.wk = a->window_k->data; mp.wv = a->window_v->data; mp.w_dtype = a->window_k->dtype;
    for (int i = 0; i < 4; ++i) {
      mp.wk_stride[i] = a->window_k->stride[i];
      mp.wv_stride[i] = a->window_v->stride[i];
    }
  }
  mp.scale_log2 = a->scale * kLog2e;
  mp.out = a->out->data; mp.out_dtype = a->out->dtype;
  for (int i = 0; i < 4; ++i) mp.out_stride[i] = a->out->stride[i];
  mp.world = a->gather ? a->gather->world : 1;
  mp.rank = a->gather ? a->gather->rank : 0;
  mp.status = reinterpret_cast<uint32_t*>(ws);
  for (int r = 0; r < TQ_MAX_PEERS; ++r) {
    mp.peer_out[r] = a->gather && r < mp.world ? a->gather->peer_out[r] : nullptr;
    mp.peer_flag[r] = a->gather && r < mp.world ? a->gather->peer_flag[r] : nullptr;
  }
  if (pl.S > 0 && (phases & TQ_PHASE_MERGE)) {
    const size_t msmem =
        (size_t)(pl.D * pl.D + 16 * pl.D + 8 * kSlotChunk * pl.D + 8 * (mp.W > 0 ? mp.W : 1)) * 4;
    // few streams: spread a chunk's heads over CTAs, up to one CTA per SM
    const int hmax = tmin(8, pl.g);
    const int64_t per = (int64_t)pl.S * pl.nch;
    const int nz = (int)tmax<int64_t>(1, tmin<int64_t>(hmax, device_sm_count() / tmax<int64_t>(per, 1)));
    const bool split = nz > 1;
    mp.hpc = split ? (hmax + nz - 1) / nz : 8;
    const unsigned mz = (unsigned)((hmax + mp.hpc - 1) / mp.hpc);
    void (*mfn)(MergeParams) =
        split ? (pl.D == 32 ? merge_kernel<32, true> : pl.D == 64 ? merge_kernel<64, true>
                                                                  : merge_kernel<128, true>)
              : (pl.D == 32 ? merge_kernel<32, false> : pl.D == 64 ? merge_kernel<64, false>
                                                                   : merge_kernel<128, false>);
    if (set_smem_attr((const void*)mfn, msmem) != TQ_OK) return TQ_ERR_CUDA;
    if (launch_result(launch_pdl(mfn, dim3((unsigned)pl.S, pl.nch, mz), dim3(kMergeThreads), msmem, st, mp),
                      "tq_decode_attn/merge") != TQ_OK)
      return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

}  // namespace tq
