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
#include "tq_prefill_tc.cuh"

#include <math.h>

namespace tq {
namespace {
using namespace pftc;

constexpr int kRows = 128;                 // query rows per CTA
constexpr int kSoftWarps = 4, kDecWarps = 8;
constexpr int kWarps = 1 + kSoftWarps + kDecWarps;
constexpr int kThreads = 32 * kWarps;      // 416
constexpr int kDecThreads = 32 * kDecWarps;
constexpr int kTmemCols = 512;
constexpr int kOCol = 256;                 // O accumulator columns
constexpr int kLCol = 384;                 // row sums of P (16 equal columns)
constexpr int kQCol = 416;                 // q' as fp16 pairs (64 columns): A of S = q' K^^T

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
    // pair tables: entries dt, dt + kDecThreads, ... with their rk (rv) copies
    for (int e = dt; e < nk; e += kDecThreads)
      put_pair_entry(lut_k, e, p.rk,
                     pack_half2(__ldg(p.kc + (e & ((1 << KB) - 1))), __ldg(p.kc + (e >> KB))));
    for (int e = dt; e < nv; e += kDecThreads)
      put_pair_entry(lut_v, e, p.rv,
                     pack_half2(__ldg(p.vc + (e & ((1 << VB) - 1))), __ldg(p.vc + (e >> VB))));
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
    const int64_t kst = row_kstart(p.kv_start, b);           // keys >= kst are seen
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
      const bool need_mask = k0 + kKeys - 1 > lim || k0 < kst;
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
            mask_keys(x0, kst - (k0 + 64 * hh), lim - (k0 + 64 * hh));
            mask_keys(x1, kst - (k0 + 64 * hh + 32), lim - (k0 + 64 * hh + 32));
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
          mask_keys(x0, kst - (k0 + 64 * hh), lim - (k0 + 64 * hh));
          mask_keys(x1, kst - (k0 + 64 * hh + 32), lim - (k0 + 64 * hh + 32));
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
    pv.pool = p.pages;
    pv.pm = p.pm;
    pv.stream = stream;
    pv.status = p.status;
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
    pv.W = p.W;
    pv.kpacked = p.n_tokens - p.W;
    const unsigned char* lk = sm + OFF_LUT + 4 * (lane & (p.rk - 1));
    const unsigned char* lv = sm + OFF_LUT + 4 * nk * p.rk + 4 * (lane & (p.rv - 1));
    const int rk4 = 4 * p.rk, rv4 = 4 * p.rv;
    const ChunkOffsets co = chunk_offsets(pv.kk, pv.part);
    // K^ runs one tile ahead of V^, so the next S MMA's operand never waits
    // behind a V^ stage that the PV MMA still holds
    HalfRegs<KB, 2> kc, kn;
    HalfRegs<VB, 2> vc, vn;
    bool ok = true;
    load_half<KB>(kc, pv, 0, 0, p.off_kn);
    decode_half<KB>(kc, lk, rk4, sm + OFF_K, co);
    if (tile_has_window(pv, 0)) window_half<2>(pv, 0, p.wk, sm + OFF_K, co);
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
        if (tile_has_window(pv, jk)) window_half<2>(pv, jk, p.wk, sm + OFF_K + sk * kStage, co);
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
      if (tile_has_window(pv, j)) window_half<2>(pv, j, p.wv, sm + OFF_V + s * kStage, co);
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
  TQ_PTC(2, 4) TQ_PTC(3, 4) TQ_PTC(2, 3) TQ_PTC(6, 4) TQ_PTC(5, 5) TQ_PTC(6, 6) TQ_PTC(5, 4)
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

// The residual window rotated once for the prefill kernels: row w of stream
// s of K (V) becomes fp16 (x R^T) with columns in K quad (V octet) order, the
// order of the decoded tiles.  grid (streams, ceil(W / kWinRows), 2: K, V),
// 128 threads; thread p computes position p of kWinRows rows from R^T and
// the rows staged in shared memory.
constexpr int kWinRows = 16;

struct WinParams {
  const void* x[2]; int dtype[2]; int64_t xs[2][4];
  int64_t Hkv, W;
  const float* rot_t;           // R^T [128][128]
  __half* out[2];               // [streams][W][128]
};

__global__ void __launch_bounds__(128) window_rotate_kernel(WinParams p) {
  extern __shared__ __align__(16) float wsm[];
  float* rt = wsm;                        // [128][128] R^T
  float* xr = rt + kD * kD;               // [kWinRows][128]
  const int which = blockIdx.z, tid = threadIdx.x;
  const int64_t s = blockIdx.x, b = s / p.Hkv, h = s % p.Hkv;
  const int64_t w0 = (int64_t)blockIdx.y * kWinRows;
  const int nrow = (int)tmin<int64_t>(kWinRows, p.W - w0);
  stage_async(rt, p.rot_t, kD * kD * 4, tid, 128);
  const int64_t* xs = p.xs[which];
  for (int i = tid; i < nrow * kD; i += 128) {
    const int r = i / kD, c = i % kD;
    xr[i] = load_elem(p.x[which], p.dtype[which],
                      b * xs[0] + h * xs[1] + (w0 + r) * xs[2] + c * xs[3]);
  }
  cp_async_wait_all();
  __syncthreads();
  const int coord = which == 0 ? k_coord(tid) : v_coord(tid);
  float acc[kWinRows];
#pragma unroll
  for (int r = 0; r < kWinRows; ++r) acc[r] = 0.f;
  for (int c = 0; c < kD; ++c) {
    const float rc = rt[c * kD + coord];
#pragma unroll
    for (int r = 0; r < kWinRows; ++r) acc[r] = fmaf(xr[r * kD + c], rc, acc[r]);
  }
  for (int r = 0; r < nrow; ++r)
    p.out[which][(s * p.W + w0 + r) * kD + tid] = __float2half_rn(acc[r]);
}

int launch_prefill_tc(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                      const tq_prefill_args* a, uint32_t* status, cudaStream_t st) {
  if (!prefill_tc_applies(G)) return 1;
  TcFn fn = tc_fn(G->key_bits, G->value_bits);
  const PageGeom g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  TcPrefillParams p;
  p.pages = c->pages;
  p.pm = page_map(c);
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
  p.kv_start = a->kv_start;
  p.W = a->window_k ? a->window_k->shape[2] : 0;
  p.wk = p.wv = nullptr;
  if (p.W > 0) {
    // rotate the window into the workspace (K, then V)
    const size_t one = tq_prefill_workspace_bytes(G, c, a) / 2;
    WinParams wp;
    const tq_tensor4* wx[2] = {a->window_k, a->window_v};
    for (int i = 0; i < 2; ++i) {
      wp.x[i] = wx[i]->data;
      wp.dtype[i] = wx[i]->dtype;
      for (int d = 0; d < 4; ++d) wp.xs[i][d] = wx[i]->stride[d];
      wp.out[i] = reinterpret_cast<__half*>(static_cast<uint8_t*>(a->workspace) + i * one);
    }
    wp.Hkv = c->streams / a->q->shape[0];
    wp.W = p.W;
    wp.rot_t = t->rot_t;
    const size_t wsmem = (size_t)(kD * kD + kWinRows * kD) * 4;
    if (set_smem_attr((const void*)window_rotate_kernel, wsmem) != TQ_OK) return TQ_ERR_CUDA;
    dim3 wgrid((unsigned)c->streams, (unsigned)((p.W + kWinRows - 1) / kWinRows), 2);
    window_rotate_kernel<<<wgrid, 128, wsmem, st>>>(wp);
    if (check_launch("tq_prefill_attn/window") != TQ_OK) return TQ_ERR_CUDA;
    p.wk = wp.out[0];
    p.wv = wp.out[1];
  }
  // pair tables: 32 copies (one per lane) where they fit, else 16 / 8
  const int nk = 1 << (2 * G->key_bits), nv = 1 << (2 * G->value_bits);
  int rk = 32, rv = 32;
  while ((nk * rk + nv * rv) * 4 > (int)kLutMax) {
    if (nk * rk >= nv * rv) rk >>= 1; else rv >>= 1;
  }
  p.rk = rk;
  p.rv = rv;
  p.status = status;
  p.pcta = P;
  p.tile_head_step = p.tile_pos_step = 0;
  if (p.Tq == 0) return TQ_OK;
  // chunks longer than one 128-row block: the 256-row kernel (engine 0 or 3)
  if (a->engine == 3 || (a->engine == 0 && p.Tq > P)) {
    const int rc = launch_prefill_tc2(p, G->key_bits, G->value_bits, B, Hq, st);
    if (rc != 1) return rc;
  }
  if (set_smem_attr((const void*)fn, SMEM_BYTES) != TQ_OK) return TQ_ERR_CUDA;
  dim3 grid((unsigned)p.nqb, (unsigned)(B * Hq / p.hc));
  fn<<<grid, kThreads, SMEM_BYTES, st>>>(p);
  return check_launch("tq_prefill_attn");
}

}  // namespace tq
