// tq_prefill_tc.cu — prefill attention straight off the packed pages on the
// 5th-generation tensor cores (tcgen05 MMAs, accumulators in tensor memory),
// for head_dim 128 with 2- to 4-bit K and V codes.  Other shapes use the
// mma.sync kernel of tq_prefill.cu.
//
// Same result as tq_prefill.cu (which gives the reference mapping):
// softmax(scale q K^T) V over the dequantised keys and values
// x^ = n (c[idx] R), computed as
//     O = softmax(q' K^T) V^,  out = O R_V
// with q' = scale log2(e) q R_K^T, K^ = n_k c_k[idx] and V^ = n_v c_v[idx].
// Columns stay in the packed orders of the page rows: K^ and q' in the quad
// order of a K row, V^ and O in the octet order of a V row.  R_K and R_V are
// R with its rows permuted into those orders, so no code is ever moved to its
// coordinate.
//
// CTA = 128 query rows (hc heads x 128/hc positions of one KV head's GQA
// group, as in tq_prefill.cu) and key tiles of 128 tokens (two pages).
// Warp roles (13 warps):
//   warp 0      owns tensor memory; one thread issues every MMA:
//               q' = Q R_K^T, then per tile S_j = q' K^_j^T and O += P_j V^_j,
//               finally OUT = O^ R_V
//   warps 1-4   softmax, one thread per query row (= tensor-memory lane):
//               reads S_j, writes P_j = exp2(S_j - m) as fp16 over the S_j
//               columns (the A operand of the PV MMA, read from tensor memory),
//               rescales O in tensor memory when the running max grows by more
//               than 8 (p <= 2^8 otherwise: exact, fp16-safe)
//   warps 5-12  decoders: codes -> fp16 K^ and V^ tiles in the 128-byte
//               swizzled layout, through pair tables (two codes -> one half2)
//               replicated across lanes; codes are read from the pages in
//               global memory with one tile of register prefetch
// Tensor memory, 512 columns: S/P double buffer at 0 and 128, O at 256, at
// 384 the row sums l = P x ones (an N = 16 MMA beside each PV MMA, so l is
// the sum of the fp16 P the PV MMA used and is rescaled with O), and at 416
// q' as fp16 pairs: both S and PV MMAs take A from tensor memory and read
// only their B tiles from shared memory.
// Shared memory: two K^ and two V^ stages of 32 KB, the pair tables (up to
// 64 KB: 32 lane copies of K4 and V4 tables), a tile of fp16 ones.  R_K and Q
// are staged in the two V stages before the first tiles; after the last,
// R_V (fp16 hi and lo terms) takes both K stages and O^ (hi and lo) both V
// stages, so the output rotation carries no fp16 rounding of O^ or R.
//
// K^ (K-major B of S = q' K^^T) and V^ (MN-major B of O = P V^) share one
// physical layout: [64-column half][128 keys][128 B], 16-byte chunks swizzled
// by key & 7.  The operand descriptors differ: K-major walks 32 B along a row
// per 16-deep MMA step, MN-major walks 16 rows (2048 B) with the halves 16 KB
// apart.
//
// Every wait is bounded; on expiry the kernel sets TQ_DEV_WAIT_TIMEOUT in the
// status word, the other roles see the abort flag, no MMA is left in flight
// and tensor memory is released.
#include "tq_common.cuh"
#include "tq_internal.h"
#include "tq_tc.cuh"

#include <math.h>

namespace tq {
namespace {

constexpr int kD = 128;
constexpr int kRows = 128;                 // query rows per CTA
constexpr int kKeys = 128;                 // keys per tile (two pages)
constexpr int kSoftWarps = 4, kDecWarps = 8;
constexpr int kWarps = 1 + kSoftWarps + kDecWarps;
constexpr int kThreads = 32 * kWarps;      // 416
constexpr int kDecThreads = 32 * kDecWarps;
constexpr int kTmemCols = 512;
constexpr int kOCol = 256;                 // O accumulator columns
constexpr int kLCol = 384;                 // row sums of P (16 equal columns)
constexpr int kQCol = 416;                 // q' as fp16 pairs (64 columns): A of S = q' K^^T
constexpr float kRescaleBits = 8.f;        // lazy rescale threshold (log2)
constexpr float kLog2e = 1.4426950408889634f;

constexpr uint32_t kHalfBytes = 16384;     // [128 rows][128 B]
constexpr uint32_t kStage = 2 * kHalfBytes;
constexpr uint32_t OFF_K = 0;
constexpr uint32_t OFF_V = OFF_K + 2 * kStage;
constexpr uint32_t OFF_LUT = OFF_V + 2 * kStage;
constexpr uint32_t kLutMax = 65536;             // K4/V4: two 256-entry tables x 32 copies
constexpr uint32_t OFF_ONES = OFF_LUT + kLutMax;   // [2][16 rows][128 B] of fp16 1.0
constexpr uint32_t OFF_RK = OFF_V;                 // R_K, before the first V^ tile
constexpr uint32_t OFF_QSTG = OFF_V + kStage;      // Q, before the second V^ tile
constexpr uint32_t OFF_OHI = OFF_V;                // O^ hi / lo after the last PV MMA
constexpr uint32_t OFF_OLO = OFF_V + kStage;
constexpr uint32_t OFF_BAR = OFF_ONES + 4096;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;   // + alignment slack

enum Bar {
  B_ROT = 0, B_QP = 1, B_KFULL = 2, B_KEMPTY = 4, B_VFULL = 6, B_VEMPTY = 8, B_SFULL = 10,
  B_PFULL = 12, B_ODONE = 14, B_OFIN = 15, B_RV = 16, B_OUT = 17, B_MMA = 18, B_PREV = 19,
  B_COUNT = 20
};

struct TcPrefillParams {
  const uint8_t* pages;
  int64_t pages_per_stream;
  int page_bytes, off_v, off_kn, off_vn;
  const __half* rot_h;          // R [128][128] fp16, row-major
  const float* rot;             // R [128][128] fp32, row-major
  const float* kc;
  const float* vc;
  const void* q; int q_dtype; int q_vec; int64_t qs[4];
  void* out; int o_dtype; int o_vec; int64_t os[4];
  int64_t Hkv, g, Tq, n_tokens;
  int hc, pshift;               // heads per CTA; log2(positions per CTA)
  int nqb;
  float qscale;                 // softmax scale * log2(e)
  int causal;
  int rk, rv;                   // pair-table replication (lanes per copy set)
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

// Scores of keys past `last` (an index into this 32-key chunk) -> -inf.
__device__ __forceinline__ void mask_keys(uint32_t (&x)[32], int64_t last) {
#pragma unroll
  for (int e = 0; e < 32; ++e)
    if (e > last) x[e] = 0xFF800000u;
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

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
        "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
        "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
               ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
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
  const uint8_t* spages;        // this stream's pages
  int page_bytes, off_v, off_kn, off_vn;
  int kk, part;
  int64_t kend;                 // keys this CTA needs
};

// One operand's codes and norms that a decoder thread needs for one tile:
// key kk of both pages, K quad / V octet pair `part`.
template <int NB>
struct HalfRegs {
  Stream<NB> c[2];
  uint32_t n[2];                // fp16 norm bits
};

template <int NB>
__device__ __forceinline__ void load_half(HalfRegs<NB>& t, const TcParamsView& pv, int j,
                                          int off_codes, int off_norm) {
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int64_t key = (int64_t)j * kKeys + p * 64 + pv.kk;
    if (key < pv.kend) {
      const uint8_t* pg = pv.spages + (int64_t)(2 * j + p) * pv.page_bytes;
      load_stream<NB>(t.c[p], pg + off_codes + pv.kk * (16 * NB) + pv.part * (4 * NB));
      t.n[p] = __ldg(reinterpret_cast<const unsigned short*>(pg + off_norm) + pv.kk);
    } else {
#pragma unroll
      for (int i = 0; i < NB; ++i) t.c[p].w[i] = 0u;
      t.n[p] = 0u;
    }
  }
}

// Decode both pages of one operand tile into the stage at `tile` (page 1's
// rows sit 64 rows = 8 KB below page 0's).
template <int NB>
__device__ __forceinline__ void decode_half(const HalfRegs<NB>& t, const unsigned char* lut,
                                            int rep4, unsigned char* tile, const ChunkOffsets& co) {
#pragma unroll
  for (int pg = 0; pg < 2; ++pg) {
    const uint32_t n2 = t.n[pg] * 0x10001u;
    decode_stream<NB>(t.c[pg], lut, rep4, *reinterpret_cast<const __half2*>(&n2),
                      tile + pg * 64 * 128, co);
  }
}

template <int KB, int VB>
__global__ void __launch_bounds__(512, 1) prefill_tc_kernel(TcPrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + B_COUNT + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = kRows / p.hc;                          // query positions per CTA
  const int qb = p.nqb - 1 - (int)blockIdx.x;          // long rows first
  const int nchunk = (int)(p.g / p.hc);
  const int64_t stream = (int64_t)blockIdx.y / nchunk;
  const int chunk = (int)((int64_t)blockIdx.y % nchunk);
  const int64_t b = stream / p.Hkv, kvh = stream % p.Hkv;
  const int64_t t_base = p.n_tokens - p.Tq;
  const int64_t qpos_max = t_base + tmin<int64_t>((int64_t)(qb + 1) * P, p.Tq) - 1;
  const int64_t kend = p.causal ? qpos_max + 1 : p.n_tokens;
  const int ntiles = (int)((kend + kKeys - 1) / kKeys);

  if (tid == 0) {
    mbar_init(&bars[B_ROT], 1);
    mbar_init(&bars[B_QP], kSoftWarps);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[B_KFULL + s], kDecWarps);
      mbar_init(&bars[B_KEMPTY + s], 1);
      mbar_init(&bars[B_VFULL + s], kDecWarps);
      mbar_init(&bars[B_VEMPTY + s], 1);
      mbar_init(&bars[B_SFULL + s], 1);
      mbar_init(&bars[B_PFULL + s], kSoftWarps);
    }
    mbar_init(&bars[B_ODONE], 1);
    mbar_init(&bars[B_PREV], 1);
    mbar_init(&bars[B_OFIN], kSoftWarps);
    mbar_init(&bars[B_RV], kDecWarps);
    mbar_init(&bars[B_OUT], 1);
    mbar_init(&bars[B_MMA], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }

  // ---- per-role setup: Q rows (softmax), R_K and the pair tables (decoders) --
  const int nk = 1 << (2 * KB), nv = 1 << (2 * VB);
  const uint32_t lut_k = sbase + OFF_LUT;
  const uint32_t lut_v = lut_k + (uint32_t)(nk * p.rk * 4);
  if (warp >= 1 && warp <= kSoftWarps) {
    // this warp's 32 rows, two rows per pass: 16 lanes x 16 bytes of a row
    const uint32_t qdst = sbase + OFF_QSTG;
    const int half = lane >> 4, c = lane & 15;
    if (p.q_vec) {
      uint4 raw[16];                            // every load in flight at once
#pragma unroll
      for (int m = 0; m < 16; ++m) {
        const int r = 32 * (warp & 3) + 2 * m + half;
        const int t = qb * P + (r & (P - 1));
        const int64_t h = kvh * p.g + (int64_t)chunk * p.hc + (r >> p.pshift);
        raw[m] = make_uint4(0, 0, 0, 0);
        if (t < p.Tq)
          raw[m] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.q) +
                                                        b * p.qs[0] + h * p.qs[1] +
                                                        (int64_t)t * p.qs[2]) + c);
      }
#pragma unroll
      for (int m = 0; m < 16; ++m)
        sts128(qdst + sw_chunk(32 * (warp & 3) + 2 * m + half, c),
               scale_chunk(raw[m], p.q_dtype, p.qscale));
    } else {
      for (int m = 0; m < 16; ++m) {
        const int r = 32 * (warp & 3) + 2 * m + half;
        const int t = qb * P + (r & (P - 1));
        const int64_t h = kvh * p.g + (int64_t)chunk * p.hc + (r >> p.pshift);
        uint32_t o[4] = {0u, 0u, 0u, 0u};
        if (t < p.Tq) {
          const int64_t base = b * p.qs[0] + h * p.qs[1] + (int64_t)t * p.qs[2];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t i = base + (int64_t)(8 * c + 2 * e) * p.qs[3];
            o[e] = pack_half2(load_elem(p.q, p.q_dtype, i) * p.qscale,
                              load_elem(p.q, p.q_dtype, i + p.qs[3]) * p.qscale);
          }
        }
        sts128(qdst + sw_chunk(r, c), make_uint4(o[0], o[1], o[2], o[3]));
      }
    }
  } else if (warp > kSoftWarps) {
    const int dt = tid - 32 * (1 + kSoftWarps);
    if (dt < 256) sts128(sbase + OFF_ONES + 16u * dt, make_uint4(0x3C003C00u, 0x3C003C00u,
                                                                 0x3C003C00u, 0x3C003C00u));
    // R_K (K-major B of q' = Q R_K^T): row i = R[k_coord(i)] -> V stage 0
    {
      constexpr int kIt = kD * 16 / kDecThreads;      // 8 chunks per thread, all in flight
      uint4 v[kIt];
#pragma unroll
      for (int m = 0; m < kIt; ++m) {
        const int it = dt + m * kDecThreads, i = it >> 4, c = it & 15;
        v[m] = __ldg(reinterpret_cast<const uint4*>(p.rot_h + k_coord(i) * kD) + c);
      }
#pragma unroll
      for (int m = 0; m < kIt; ++m) {
        const int it = dt + m * kDecThreads;
        sts128(sbase + OFF_RK + sw_chunk(it >> 4, it & 15), v[m]);
      }
    }
    // pair tables: one entry per thread, its rk (rv) copies written 16 bytes
    // at a time (rk, rv >= 8 and nk, nv <= 256 = decoder threads)
    if (dt < nk) {
      const uint32_t v = pack_half2(__ldg(p.kc + (dt & ((1 << KB) - 1))), __ldg(p.kc + (dt >> KB)));
      const uint4 v4 = make_uint4(v, v, v, v);
      for (int c = 0; c < p.rk; c += 4) sts128(lut_k + 4u * (uint32_t)(dt * p.rk + c), v4);
    }
    if (dt < nv) {
      const uint32_t v = pack_half2(__ldg(p.vc + (dt & ((1 << VB) - 1))), __ldg(p.vc + (dt >> VB)));
      const uint4 v4 = make_uint4(v, v, v, v);
      for (int c = 0; c < p.rv; c += 4) sts128(lut_v + 4u * (uint32_t)(dt * p.rv + c), v4);
    }
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  constexpr uint32_t idesc_kk = tc::idesc_f16_f32(kRows, 128);            // A, B K-major
  constexpr uint32_t idesc_kmn = tc::idesc_f16_f32(kRows, 128) | (1u << 16);   // B MN-major
  constexpr uint32_t idesc_l = tc::idesc_f16_f32(kRows, 16);                   // P x ones

  if (warp == 0) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      bool ok = true;
      // q' = Q R_K^T into columns 0..127
#pragma unroll
      for (int st = 0; st < 8; ++st) {
        const uint32_t off = (uint32_t)((st >> 2) * kHalfBytes + (st & 3) * 32);
        umma_ss(tmem, tc::sdesc_kmajor_sw128(sbase + OFF_QSTG + off),
                      tc::sdesc_kmajor_sw128(sbase + OFF_RK + off), idesc_kk, st ? 1u : 0u);
      }
      tc::umma_commit(&bars[B_ROT]);
      ok = wait_or_abort(&bars[B_QP], 0u, abort_flag, p.status);
      tc::tc_fence_after();
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!wait_or_abort(&bars[B_KFULL + s], (uint32_t)((j >> 1) & 1), abort_flag, p.status))
          return false;
        tc::tc_fence_after();
        const uint32_t kbase = sbase + OFF_K + s * kStage;
#pragma unroll
        for (int st = 0; st < 8; ++st) {
          const uint32_t off = (uint32_t)((st >> 2) * kHalfBytes + (st & 3) * 32);
          umma_ts(tmem + s * 128, tmem + kQCol + 8 * st, tc::sdesc_kmajor_sw128(kbase + off),
                  idesc_kk, st ? 1u : 0u);
        }
        tc::umma_commit(&bars[B_KEMPTY + s]);
        tc::umma_commit(&bars[B_SFULL + s]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int s = j & 1;
        const uint32_t par = (uint32_t)((j >> 1) & 1);
        if (!wait_or_abort(&bars[B_PFULL + s], par, abort_flag, p.status) ||
            !wait_or_abort(&bars[B_VFULL + s], par, abort_flag, p.status))
          return false;
        tc::tc_fence_after();
        const uint32_t vbase = sbase + OFF_V + s * kStage;
#pragma unroll
        for (int st = 0; st < 8; ++st)
          umma_ts(tmem + kOCol, tmem + s * 128 + 8 * st,
                  sdesc_mnmajor_sw128(vbase + st * 2048, kHalfBytes), idesc_kmn,
                  (j | st) ? 1u : 0u);
#pragma unroll
        for (int st = 0; st < 8; ++st)
          umma_ts(tmem + kLCol, tmem + s * 128 + 8 * st,
                  tc::sdesc_kmajor_sw128(sbase + OFF_ONES + (st >> 2) * 2048 + (st & 3) * 32),
                  idesc_l, (j | st) ? 1u : 0u);
        tc::umma_commit(&bars[B_VEMPTY + s]);
        if (j == ntiles - 2) tc::umma_commit(&bars[B_PREV]);
        if (j == ntiles - 1) tc::umma_commit(&bars[B_ODONE]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && ntiles > 1) ok = issue_s(1);
      for (int j = 0; ok && j < ntiles; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < ntiles) ok = issue_s(j + 2);
      }
      // OUT = O^ R_V into columns 0..127
      if (ok && wait_or_abort(&bars[B_OFIN], 0u, abort_flag, p.status) &&
          wait_or_abort(&bars[B_RV], 0u, abort_flag, p.status)) {
        tc::tc_fence_after();
        // O^hi R_V,hi + O^lo R_V,hi + O^hi R_V,lo
#pragma unroll
        for (int term = 0; term < 3; ++term) {
          const uint32_t abase = sbase + (term == 1 ? OFF_OLO : OFF_OHI);
          const uint32_t bbase = sbase + OFF_K + (term == 2 ? kStage : 0u);
#pragma unroll
          for (int st = 0; st < 8; ++st) {
            const uint32_t off = (uint32_t)((st >> 2) * kHalfBytes + (st & 3) * 32);
            umma_ss(tmem, tc::sdesc_kmajor_sw128(abase + off),
                    sdesc_mnmajor_sw128(bbase + st * 2048, kHalfBytes), idesc_kmn,
                    (term | st) ? 1u : 0u);
          }
        }
        tc::umma_commit(&bars[B_OUT]);
      }
      // never leave with an MMA in flight
      tc::umma_commit(&bars[B_MMA]);
      mbar_wait_bounded(&bars[B_MMA], 0u, 16u);
    }
    __syncwarp();
  } else if (warp <= kSoftWarps) {
    // ================================================================ softmax
    const int quarter = warp & 3;
    const int r = 32 * quarter + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
    const int pl = r & (P - 1), hl = r >> p.pshift;
    const int t = qb * P + pl;
    const bool valid = t < p.Tq;
    const int64_t qpos = valid ? t_base + t : qpos_max;
    const int64_t lim = p.causal ? qpos : p.n_tokens - 1;    // keys <= lim are seen
    bool ok = __all_sync(0xffffffffu, wait_or_abort(&bars[B_ROT], 0u, abort_flag, p.status));
    if (ok) {
      // q' (fp32, K order) -> fp16 pairs in tensor memory (A of the S MMA)
      tc::tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; c += 2) {
        uint32_t x0[32], x1[32];
        tc::tmem_ld_x32(tl + 32 * c, x0);
        tc::tmem_ld_x32(tl + 32 * c + 32, x1);
        tmem_ld_wait(x0);
        tmem_ld_wait(x1);
        uint32_t h[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          h[e] = pack_half2(__uint_as_float(x0[2 * e]), __uint_as_float(x0[2 * e + 1]));
          h[16 + e] = pack_half2(__uint_as_float(x1[2 * e]), __uint_as_float(x1[2 * e + 1]));
        }
        tc::tmem_st_x32(tl + kQCol + 16 * c, h);
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cta(&bars[B_QP]);
    }
    float m = -INFINITY;
    for (int j = 0; ok && j < ntiles; ++j) {
      const int s = j & 1;
      ok = __all_sync(0xffffffffu,
                      wait_or_abort(&bars[B_SFULL + s], (uint32_t)((j >> 1) & 1), abort_flag,
                                    p.status));
      if (!ok) break;
      tc::tc_fence_after();
      const int64_t k0 = (int64_t)j * kKeys;
      const bool need_mask = k0 + kKeys - 1 > lim;
      const uint32_t scol = tl + s * 128;
      // pass 1: row max (four independent 3-input chains)
      float mx;
      {
        float a0 = -INFINITY, a1 = -INFINITY, a2 = -INFINITY, a3 = -INFINITY;
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t x0[32], x1[32];
          tc::tmem_ld_x32(scol + 64 * hh, x0);
          tc::tmem_ld_x32(scol + 64 * hh + 32, x1);
          tmem_ld_wait(x0);
          tmem_ld_wait(x1);
          if (need_mask) {
            mask_keys(x0, lim - (k0 + 64 * hh));
            mask_keys(x1, lim - (k0 + 64 * hh + 32));
          }
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            a0 = fmax3(a0, __uint_as_float(x0[e]), __uint_as_float(x0[e + 1]));
            a1 = fmax3(a1, __uint_as_float(x0[e + 2]), __uint_as_float(x0[e + 3]));
            a2 = fmax3(a2, __uint_as_float(x0[e + 4]), __uint_as_float(x0[e + 5]));
            a3 = fmax3(a3, __uint_as_float(x0[e + 6]), __uint_as_float(x0[e + 7]));
            a0 = fmax3(a0, __uint_as_float(x1[e]), __uint_as_float(x1[e + 1]));
            a1 = fmax3(a1, __uint_as_float(x1[e + 2]), __uint_as_float(x1[e + 3]));
            a2 = fmax3(a2, __uint_as_float(x1[e + 4]), __uint_as_float(x1[e + 5]));
            a3 = fmax3(a3, __uint_as_float(x1[e + 6]), __uint_as_float(x1[e + 7]));
          }
        }
        mx = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
      }
      const float m_new = fmaxf(m, mx);
      const bool resc = m != -INFINITY && m_new > m + kRescaleBits;
      const float f = resc ? fast_exp2(m - m_new) : 1.f;
      if (m == -INFINITY || resc) m = m_new;
      const float bias = m == -INFINITY ? 0.f : m;
      const uint64_t nbias2 = (uint64_t)__float_as_uint(-bias) * 0x100000001ull;
      // pass 2: P = exp2(S - m) as fp16 pairs over the S columns (masked
      // scores are -inf: p = 0); the row sum comes from the P x ones MMA
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t x0[32], x1[32];
        tc::tmem_ld_x32(scol + 64 * hh, x0);
        tc::tmem_ld_x32(scol + 64 * hh + 32, x1);
        tmem_ld_wait(x0);
        tmem_ld_wait(x1);
        if (need_mask) {
          mask_keys(x0, lim - (k0 + 64 * hh));
          mask_keys(x1, lim - (k0 + 64 * hh + 32));
        }
        uint32_t h[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          h[e] = exp2_pair(x0[2 * e], x0[2 * e + 1], nbias2);
          h[16 + e] = exp2_pair(x1[2 * e], x1[2 * e + 1], nbias2);
        }
        tc::tmem_st_x32(scol + 32 * hh, h);
      }
      // rescaling O needs O += P V^ of tile j - 1 complete.  Commits complete
      // in issue order and S_{j+1} was issued after PV_{j-1}, so S_{j+1}
      // complete (a phase this warp waits for next anyway; it cannot advance
      // again before P_{j+1} exists) implies it; the last tile waits for the
      // commit that follows PV_{j-1}.
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        if (j + 1 < ntiles)
          ok = wait_or_abort(&bars[B_SFULL + ((j + 1) & 1)], (uint32_t)(((j + 1) >> 1) & 1),
                             abort_flag, p.status);
        else
          ok = wait_or_abort(&bars[B_PREV], 0u, abort_flag, p.status);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc::tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t x[32];
            tc::tmem_ld_x32(tl + kOCol + 32 * c, x);
            tmem_ld_wait(x);
#pragma unroll
            for (int e = 0; e < 32; ++e) x[e] = __float_as_uint(__uint_as_float(x[e]) * f);
            tc::tmem_st_x32(tl + kOCol + 32 * c, x);
          }
          {
            uint32_t x[32];
            tmem_ld_x16(tl + kLCol, x);
            tmem_ld_wait(x);
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = __float_as_uint(__uint_as_float(x[e]) * f);
            tmem_st_x16(tl + kLCol, reinterpret_cast<const uint32_t(&)[16]>(x));
          }
        }
      }
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (ok && lane == 0) tc::mbar_arrive_cta(&bars[B_PFULL + s]);
    }
    // O^ = O / l (V order) -> fp16 hi (over q') + lo (V stage 0; every PV MMA
    // is complete) A operands
    if (ok)
      ok = __all_sync(0xffffffffu, wait_or_abort(&bars[B_ODONE], 0u, abort_flag, p.status));
    if (ok) {
      tc::tc_fence_after();
      float l;
      {
        uint32_t x[32];
        tmem_ld_x16(tl + kLCol, x);
        tmem_ld_wait(x);
        l = __uint_as_float(x[0]);
      }
      const float il = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        tc::tmem_ld_x32(tl + kOCol + 32 * c, x);
        tmem_ld_wait(x);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t h[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a = __uint_as_float(x[8 * q + 2 * e]) * il;
            const float b = __uint_as_float(x[8 * q + 2 * e + 1]) * il;
            h[e] = pack_half2(a, b);
            const __half2 hh = *reinterpret_cast<const __half2*>(&h[e]);
            lo[e] = pack_half2(a - __low2float(hh), b - __high2float(hh));
          }
          sts128(sbase + OFF_OHI + sw_chunk(r, 4 * c + q), make_uint4(h[0], h[1], h[2], h[3]));
          sts128(sbase + OFF_OLO + sw_chunk(r, 4 * c + q), make_uint4(lo[0], lo[1], lo[2], lo[3]));
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cta(&bars[B_OFIN]);
      ok = __all_sync(0xffffffffu, wait_or_abort(&bars[B_OUT], 0u, abort_flag, p.status));
    }
    if (ok) {
      tc::tc_fence_after();
      const int64_t h = kvh * p.g + (int64_t)chunk * p.hc + hl;
      const int64_t base = b * p.os[0] + h * p.os[1] + (int64_t)t * p.os[2];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        tc::tmem_ld_x32(tl + 32 * c, x);
        tmem_ld_wait(x);
        if (!valid) continue;
        if (p.o_vec) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + base) + 4 * c;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(x[8 * q + 2 * e]);
              const float hi = __uint_as_float(x[8 * q + 2 * e + 1]);
              if (p.o_dtype == TQ_F16) {
                h[e] = pack_half2(lo, hi);
              } else {
                __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
                h[e] = *reinterpret_cast<uint32_t*>(&v);
              }
            }
            dst[q] = make_uint4(h[0], h[1], h[2], h[3]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            store_elem(p.out, p.o_dtype, base + (int64_t)(32 * c + e) * p.os[3],
                       __uint_as_float(x[e]));
        }
      }
    }
  } else {
    // ================================================================ decoders
    const int dt = tid - 32 * (1 + kSoftWarps);
    TcParamsView pv;
    pv.spages = p.pages + stream * p.pages_per_stream * (int64_t)p.page_bytes;
    pv.page_bytes = p.page_bytes;
    pv.off_v = p.off_v;
    pv.off_kn = p.off_kn;
    pv.off_vn = p.off_vn;
    // lane -> (key, part): a warp covers 8 keys x 4 parts (512 contiguous
    // code bytes per load); within each 8-lane group of a 16-byte store the
    // 8 lanes hit 8 distinct 16-byte slots of the swizzled rows (parts 0 and
    // 2 of one key would share a slot in the two 64-column halves)
    {
      const int G = lane >> 3, u = lane & 7, part = u & 3;
      const int klo = ((u >> 2) ^ ((((part >> 1) ^ G) & 1) << 1)) | ((G >> 1) << 2);
      pv.kk = 8 * (dt >> 5) + klo;
      pv.part = part;
    }
    pv.kend = kend;
    const unsigned char* lk = sm + OFF_LUT + 4 * (lane & (p.rk - 1));
    const unsigned char* lv = sm + OFF_LUT + 4 * nk * p.rk + 4 * (lane & (p.rv - 1));
    const int rk4 = 4 * p.rk, rv4 = 4 * p.rv;
    const ChunkOffsets co = chunk_offsets(pv.kk, pv.part);
    // K^ runs one tile ahead of V^, so the next S MMA's operand never waits
    // behind a V^ stage that the PV MMA still holds
    HalfRegs<KB> kc, kn;
    HalfRegs<VB> vc, vn;
    bool ok = true;
    load_half<KB>(kc, pv, 0, 0, p.off_kn);
    decode_half<KB>(kc, lk, rk4, sm + OFF_K, co);
    tc::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) tc::mbar_arrive_cta(&bars[B_KFULL]);
    if (ntiles > 1) load_half<KB>(kc, pv, 1, 0, p.off_kn);
    load_half<VB>(vc, pv, 0, p.off_v, p.off_vn);
    for (int j = 0; j < ntiles; ++j) {
      if (j + 2 < ntiles) load_half<KB>(kn, pv, j + 2, 0, p.off_kn);
      if (j + 1 < ntiles) load_half<VB>(vn, pv, j + 1, p.off_v, p.off_vn);
      if (j + 1 < ntiles) {
        // K^ of tile j + 1: the S MMA of tile j - 1 has read this stage
        const int jk = j + 1, sk = jk & 1;
        if (jk >= 2)
          ok = wait_or_abort(&bars[B_KEMPTY + sk], (uint32_t)(((jk >> 1) - 1) & 1), abort_flag,
                             p.status);
        if (!__all_sync(0xffffffffu, ok)) break;
        decode_half<KB>(kc, lk, rk4, sm + OFF_K + sk * kStage, co);
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cta(&bars[B_KFULL + sk]);
      }
      // V^ of tile j: the PV MMA of tile j - 2 has read this stage
      const int s = j & 1;
      if (j >= 2)
        ok = wait_or_abort(&bars[B_VEMPTY + s], (uint32_t)(((j >> 1) - 1) & 1), abort_flag,
                           p.status);
      else   // tiles 0 and 1: R_K and Q sit in the V stages until q' = Q R_K^T is done
        ok = wait_or_abort(&bars[B_ROT], 0u, abort_flag, p.status);
      if (!__all_sync(0xffffffffu, ok)) break;
      decode_half<VB>(vc, lv, rv4, sm + OFF_V + s * kStage, co);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cta(&bars[B_VFULL + s]);
      kc = kn;
      vc = vn;
    }
    // R_V (MN-major B of OUT = O^ R_V): row i = R[v_coord(i)], fp16 hi in K
    // stage 0 and lo = R - hi in K stage 1, once the last S MMAs that read
    // those stages are complete.  The fp32 rows are fetched first (all loads
    // in flight), then the stages are awaited.
    constexpr int kIt = kD * 16 / kDecThreads;            // 8 chunks per thread
    float4 rv[kIt][2];
#pragma unroll
    for (int m = 0; m < kIt; ++m) {
      const int it = dt + m * kDecThreads, i = it >> 4, c = it & 15;
      const float4* src = reinterpret_cast<const float4*>(p.rot + v_coord(i) * kD + 8 * c);
      rv[m][0] = __ldg(src);
      rv[m][1] = __ldg(src + 1);
    }
    if (ok) {
      const int j0 = (ntiles - 1) & ~1;                   // last tile in stage 0
      ok = wait_or_abort(&bars[B_KEMPTY], (uint32_t)((j0 >> 1) & 1), abort_flag, p.status);
      if (ok && ntiles >= 2) {
        const int j1 = (ntiles - 1) & 1 ? ntiles - 1 : ntiles - 2;   // last tile in stage 1
        ok = wait_or_abort(&bars[B_KEMPTY + 1], (uint32_t)((j1 >> 1) & 1), abort_flag, p.status);
      }
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
#pragma unroll
      for (int m = 0; m < kIt; ++m) {
        const int it = dt + m * kDecThreads, i = it >> 4, c = it & 15;
        const float v[8] = {rv[m][0].x, rv[m][0].y, rv[m][0].z, rv[m][0].w,
                            rv[m][1].x, rv[m][1].y, rv[m][1].z, rv[m][1].w};
        uint32_t h[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = pack_half2(v[2 * e], v[2 * e + 1]);
          const __half2 hh = *reinterpret_cast<const __half2*>(&h[e]);
          lo[e] = pack_half2(v[2 * e] - __low2float(hh), v[2 * e + 1] - __high2float(hh));
        }
        sts128(sbase + OFF_K + sw_chunk(i, c), make_uint4(h[0], h[1], h[2], h[3]));
        sts128(sbase + OFF_K + kStage + sw_chunk(i, c), make_uint4(lo[0], lo[1], lo[2], lo[3]));
      }
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cta(&bars[B_RV]);
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

using TcFn = void (*)(TcPrefillParams);

TcFn tc_fn(int kb, int vb) {
#define TQ_PTC(K, V) if (kb == K && vb == V) return prefill_tc_kernel<K, V>;
  TQ_PTC(4, 2) TQ_PTC(4, 4) TQ_PTC(3, 3) TQ_PTC(2, 2) TQ_PTC(3, 2) TQ_PTC(4, 3)
  TQ_PTC(2, 4) TQ_PTC(3, 4) TQ_PTC(2, 3)
#undef TQ_PTC
  return nullptr;
}

bool vec_ok(const tq_tensor4* x) {
  if (x->dtype != TQ_BF16 && x->dtype != TQ_F16) return false;
  if (x->stride[3] != 1 || reinterpret_cast<uintptr_t>(x->data) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (x->stride[i] % 8) return false;
  return true;
}

}  // namespace

bool prefill_tc_applies(const tq_geom* G) {
  return G->head_dim == kD && tc_fn(G->key_bits, G->value_bits) != nullptr;
}

int launch_prefill_tc(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                      const tq_prefill_args* a, uint32_t* status, cudaStream_t st) {
  if (!prefill_tc_applies(G)) return 1;
  TcFn fn = tc_fn(G->key_bits, G->value_bits);
  const PageGeom g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  TcPrefillParams p;
  p.pages = c->pages;
  p.pages_per_stream = c->pages_per_stream;
  p.page_bytes = g.page_bytes;
  p.off_v = g.off_v;
  p.off_kn = g.off_kn;
  p.off_vn = g.off_vn;
  p.rot_h = reinterpret_cast<const __half*>(t->rot_f16);
  p.rot = t->rot;
  p.kc = t->k_centroids;
  p.vc = t->v_centroids;
  p.q = a->q->data; p.q_dtype = a->q->dtype; p.q_vec = vec_ok(a->q);
  p.out = a->out->data; p.o_dtype = a->out->dtype; p.o_vec = vec_ok(a->out);
  for (int i = 0; i < 4; ++i) { p.qs[i] = a->q->stride[i]; p.os[i] = a->out->stride[i]; }
  const int64_t B = a->q->shape[0], Hq = a->q->shape[1];
  p.Hkv = c->streams / B;
  p.g = Hq / p.Hkv;
  p.hc = p.g % 8 == 0 ? 8 : p.g % 4 == 0 ? 4 : p.g % 2 == 0 ? 2 : 1;
  const int P = kRows / p.hc;
  p.pshift = 0;
  while ((1 << p.pshift) < P) ++p.pshift;
  p.Tq = a->q->shape[2];
  p.n_tokens = a->n_tokens;
  p.nqb = (int)((p.Tq + P - 1) / P);
  p.qscale = a->scale * kLog2e;
  p.causal = a->causal;
  // pair tables: 32 copies (one per lane) where they fit, else 16 / 8
  const int nk = 1 << (2 * G->key_bits), nv = 1 << (2 * G->value_bits);
  int rk = 32, rv = 32;
  while ((nk * rk + nv * rv) * 4 > (int)kLutMax) {
    if (nk * rk >= nv * rv) rk >>= 1; else rv >>= 1;
  }
  p.rk = rk;
  p.rv = rv;
  p.status = status;
  if (p.Tq == 0) return TQ_OK;
  if (set_smem_attr((const void*)fn, SMEM_BYTES) != TQ_OK) return TQ_ERR_CUDA;
  dim3 grid((unsigned)p.nqb, (unsigned)(B * Hq / p.hc));
  fn<<<grid, kThreads, SMEM_BYTES, st>>>(p);
  return check_launch("tq_prefill_attn");
}

}  // namespace tq
