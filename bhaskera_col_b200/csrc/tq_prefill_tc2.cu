// tq_prefill_tc2.cu — tcgen05 prefill attention with 256 query rows per CTA:
// two 128-row query tiles (A and B) share every decoded K^ / V^ tile, so the
// decode work per flop halves, and their two softmax warp groups alternate on
// the tensor core (while one group turns S into P, the MMA issuer runs the
// other tile's PV and next S).
//
// Math and layouts as in tq_prefill_tc.cu (see tq_prefill_tc.cuh):
//     O = softmax(q' K^T) V^,  out = O R_V,  q' = scale log2(e) q R_K^T.
// Rows: with hc >= 2 heads per CTA, tile X holds heads X hc/2 .. X hc/2 +
// hc/2 - 1 at the CTA's 256/hc positions (both tiles need the same keys);
// with hc = 1 tile X holds positions 128 X .. 128 X + 127 of the head.
//
// Warp roles (17 warps):
//   warp 0      owns tensor memory; one thread issues every MMA in the order
//               S_A(0) S_B(0), then per tile j: PV_A(j) S_A(j+1) PV_B(j)
//               S_B(j+1); finally OUT_X = O^_X R_V
//   warps 1-4   softmax of tile A, warps 5-8 softmax of tile B, one thread
//               per query row (tensor-memory lane): S_X(j) -> P_X(j) as fp16
//               pairs over the S_X columns, row sums l in registers (sums of
//               the fp16 P the PV MMA uses), lazy O_X rescale in tensor memory
//   warps 9-16  decoders (K^ one tile ahead of V^, two rows per thread: the
//               same key row of both pages; eight warps so that decoding, not
//               issue latency, sets their pace)
// Tensor memory (512 columns): S_A 0, S_B 128, O_A 256, O_B 384.  With one S
// buffer per tile, S_X(j) complete implies PV_X(j-1) complete (issued
// before it), so a rescale of O_X needs no extra wait.
// Shared memory: Q_A / Q_B staged and replaced by q'_A / q'_B (fp16 A of S),
// two K^ and two V^ stages, the pair tables.  R_K sits in V stage 0 before
// the first V^ tile; after the last MMA of the loop R_V hi / lo replace q'_A
// / q'_B, O^_A hi / lo the K stages and O^_B hi / lo the V stages.
//
// Every wait is bounded; on expiry the kernel sets TQ_DEV_WAIT_TIMEOUT in the
// status word, the other roles see the abort flag, no MMA is left in flight
// and tensor memory is released.
#include "tq_prefill_tc.cuh"

#include <math.h>

namespace tq {
namespace {
using namespace pftc;

constexpr int kSoftWarps = 8;              // 4 per query tile
constexpr int kDecWarps = 8;
constexpr int kWarps = 1 + kSoftWarps + kDecWarps;
constexpr int kThreads = 32 * kWarps;      // 544
constexpr int kDecThreads = 32 * kDecWarps;
constexpr int kTmemCols = 512;

constexpr uint32_t OFF_QA = 0;
constexpr uint32_t OFF_QB = kStage;
constexpr uint32_t OFF_K = 2 * kStage;
constexpr uint32_t OFF_V = 4 * kStage;
constexpr uint32_t OFF_LUT = 6 * kStage;
constexpr uint32_t kLutMax = 32768;
constexpr uint32_t OFF_BAR = OFF_LUT + kLutMax;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;   // + alignment slack

enum Bar {
  B_ROT = 0, B_QP = 1, B_KFULL = 3, B_KEMPTY = 5, B_VFULL = 7, B_VEMPTY = 9, B_SFULL = 11,
  B_PFULL = 13, B_ODONE = 15, B_OFIN = 16, B_RV = 17, B_OUT = 18, B_MMA = 19, B_COUNT = 20
};

// l0 += lo(h), l1 += hi(h) for the two fp16 halves of h (exact fp32 adds).
__device__ __forceinline__ void sum_f16x2(uint32_t h, float& l0, float& l1) {
  asm("{\n .reg .b16 lo, hi, one;\n mov.b16 one, 0x3C00;\n mov.b32 {lo, hi}, %2;\n"
      " fma.rn.f32.f16 %0, lo, one, %0;\n fma.rn.f32.f16 %1, hi, one, %1;\n}"
      : "+f"(l0), "+f"(l1) : "r"(h));
}

// Query row of tile X, lane row rr: (head within the CTA's heads, position).
struct RowId { int head; int pos; };
__device__ __forceinline__ RowId row_id(const TcPrefillParams& p, int qb, int X, int rr) {
  RowId r;
  r.head = X * p.tile_head_step + (rr >> p.pshift);
  r.pos = qb * p.pcta + X * p.tile_pos_step + (rr & ((1 << p.pshift) - 1));
  return r;
}

template <int KB, int VB>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc2_kernel(TcPrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const uint32_t sbase = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + B_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + B_COUNT + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = p.nqb - 1 - (int)blockIdx.x;          // long rows first
  const int nchunk = (int)(p.g / p.hc);
  const int64_t stream = (int64_t)blockIdx.y / nchunk;
  const int chunk = (int)((int64_t)blockIdx.y % nchunk);
  const int64_t b = stream / p.Hkv, kvh = stream % p.Hkv;
  const int64_t t_base = p.n_tokens - p.Tq;
  const int64_t qpos_max = t_base + tmin<int64_t>((int64_t)(qb + 1) * p.pcta, p.Tq) - 1;
  const int64_t kend = p.causal ? qpos_max + 1 : p.n_tokens;
  const int ntiles = (int)((kend + kKeys - 1) / kKeys);

  if (tid == 0) {
    mbar_init(&bars[B_ROT], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[B_QP + s], 4);
      mbar_init(&bars[B_KFULL + s], kDecWarps);
      mbar_init(&bars[B_KEMPTY + s], 1);
      mbar_init(&bars[B_VFULL + s], kDecWarps);
      mbar_init(&bars[B_VEMPTY + s], 1);
      mbar_init(&bars[B_SFULL + s], 1);
      mbar_init(&bars[B_PFULL + s], 4);
    }
    mbar_init(&bars[B_ODONE], 1);
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

  // ---- setup: Q rows (softmax groups), R_K and the pair tables (decoders) ----
  const int nk = 1 << (2 * KB), nv = 1 << (2 * VB);
  if (warp >= 1 && warp <= kSoftWarps) {
    // this warp's 32 rows of its tile, two rows per pass: 16 lanes x 16 bytes
    const int X = (warp - 1) >> 2;
    const uint32_t qdst = sbase + OFF_QA + X * kStage;
    const int half = lane >> 4, c = lane & 15;
    uint4 raw4[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int rr = 32 * (warp & 3) + 2 * m + half;
      const RowId id = row_id(p, qb, X, rr);
      const int64_t h = kvh * p.g + (int64_t)chunk * p.hc + id.head;
      raw4[m] = make_uint4(0, 0, 0, 0);
      if (id.pos < p.Tq) {
        const int64_t base = b * p.qs[0] + h * p.qs[1] + (int64_t)id.pos * p.qs[2];
        if (p.q_vec) {
          raw4[m] = __ldg(reinterpret_cast<const uint4*>(
                              reinterpret_cast<const uint16_t*>(p.q) + base) + c);
        } else {
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t i = base + (int64_t)(8 * c + 2 * e) * p.qs[3];
            o[e] = pack_half2(load_elem(p.q, p.q_dtype, i) * p.qscale,
                              load_elem(p.q, p.q_dtype, i + p.qs[3]) * p.qscale);
          }
          raw4[m] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const int rr = 32 * (warp & 3) + 2 * m + half;
      sts128(qdst + sw_chunk(rr, c), p.q_vec ? scale_chunk(raw4[m], p.q_dtype, p.qscale) : raw4[m]);
    }
  } else if (warp > kSoftWarps) {
    const int dt = tid - 32 * (1 + kSoftWarps);
    // R_K (K-major B of q' = Q R_K^T): row i = R[k_coord(i)] -> V stage 0
    {
      constexpr int kIt = kD * 16 / kDecThreads;      // 16 chunks per thread, all in flight
      uint4 v[kIt];
#pragma unroll
      for (int m = 0; m < kIt; ++m) {
        const int it = dt + m * kDecThreads, i = it >> 4, c = it & 15;
        v[m] = __ldg(reinterpret_cast<const uint4*>(p.rot_h + k_coord(i) * kD) + c);
      }
#pragma unroll
      for (int m = 0; m < kIt; ++m) {
        const int it = dt + m * kDecThreads;
        sts128(sbase + OFF_V + sw_chunk(it >> 4, it & 15), v[m]);
      }
    }
    // pair tables: entries dt, dt + 128, ... with their rk (rv) copies
    const uint32_t lut_k = sbase + OFF_LUT;
    const uint32_t lut_v = lut_k + (uint32_t)(nk * p.rk * 4);
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

  constexpr uint32_t idesc_kk = tc::idesc_f16_f32(128, 128);                 // A, B K-major
  constexpr uint32_t idesc_kmn = tc::idesc_f16_f32(128, 128) | (1u << 16);    // B MN-major

  if (warp == 0) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      bool ok = true;
      // q'_X = Q_X R_K^T into S_X's columns
#pragma unroll
      for (int X = 0; X < 2; ++X)
#pragma unroll
        for (int st = 0; st < 8; ++st) {
          const uint32_t off = (uint32_t)((st >> 2) * kHalfBytes + (st & 3) * 32);
          umma_ss(tmem + 128 * X, tc::sdesc_kmajor_sw128(sbase + OFF_QA + X * kStage + off),
                  tc::sdesc_kmajor_sw128(sbase + OFF_V + off), idesc_kk, st ? 1u : 0u);
        }
      tc::umma_commit(&bars[B_ROT]);
      auto issue_s = [&](int X, int j) -> bool {
        const int s = j & 1;
        if (X == 0 &&
            !wait_or_abort(&bars[B_KFULL + s], (uint32_t)((j >> 1) & 1), abort_flag, p.status))
          return false;
        tc::tc_fence_after();
        const uint32_t kbase = sbase + OFF_K + s * kStage;
        const uint32_t qbase = sbase + OFF_QA + X * kStage;
#pragma unroll
        for (int st = 0; st < 8; ++st) {
          const uint32_t off = (uint32_t)((st >> 2) * kHalfBytes + (st & 3) * 32);
          umma_ss(tmem + 128 * X, tc::sdesc_kmajor_sw128(qbase + off),
                  tc::sdesc_kmajor_sw128(kbase + off), idesc_kk, st ? 1u : 0u);
        }
        tc::umma_commit(&bars[B_SFULL + X]);
        if (X == 1) tc::umma_commit(&bars[B_KEMPTY + s]);   // both S MMAs have read K^_j
        return true;
      };
      auto issue_pv = [&](int X, int j) -> bool {
        const int s = j & 1;
        if (!wait_or_abort(&bars[B_PFULL + X], (uint32_t)(j & 1), abort_flag, p.status))
          return false;
        if (X == 0 &&
            !wait_or_abort(&bars[B_VFULL + s], (uint32_t)((j >> 1) & 1), abort_flag, p.status))
          return false;
        tc::tc_fence_after();
        const uint32_t vbase = sbase + OFF_V + s * kStage;
#pragma unroll
        for (int st = 0; st < 8; ++st)
          umma_ts(tmem + 256 + 128 * X, tmem + 128 * X + 8 * st,
                  sdesc_mnmajor_sw128(vbase + st * 2048, kHalfBytes), idesc_kmn,
                  (j | st) ? 1u : 0u);
        if (X == 1) {
          tc::umma_commit(&bars[B_VEMPTY + s]);          // both PV MMAs have read V^_j
          if (j == ntiles - 1) tc::umma_commit(&bars[B_ODONE]);
        }
        return true;
      };
      ok = wait_or_abort(&bars[B_QP], 0u, abort_flag, p.status) && issue_s(0, 0) &&
           wait_or_abort(&bars[B_QP + 1], 0u, abort_flag, p.status) && issue_s(1, 0);
      for (int j = 0; ok && j < ntiles; ++j) {
        ok = issue_pv(0, j);
        if (ok && j + 1 < ntiles) ok = issue_s(0, j + 1);
        if (ok) ok = issue_pv(1, j);
        if (ok && j + 1 < ntiles) ok = issue_s(1, j + 1);
      }
      // OUT_X = O^_X R_V into S_X's columns: O^hi R_V,hi + O^lo R_V,hi + O^hi R_V,lo
      if (ok && wait_or_abort(&bars[B_OFIN], 0u, abort_flag, p.status) &&
          wait_or_abort(&bars[B_RV], 0u, abort_flag, p.status)) {
        tc::tc_fence_after();
#pragma unroll
        for (int X = 0; X < 2; ++X) {
          const uint32_t ohi = sbase + (X == 0 ? OFF_K : OFF_V);
#pragma unroll
          for (int term = 0; term < 3; ++term) {
            const uint32_t abase = ohi + (term == 1 ? kStage : 0u);
            const uint32_t bbase = sbase + (term == 2 ? OFF_QB : OFF_QA);
#pragma unroll
            for (int st = 0; st < 8; ++st) {
              const uint32_t off = (uint32_t)((st >> 2) * kHalfBytes + (st & 3) * 32);
              umma_ss(tmem + 128 * X, tc::sdesc_kmajor_sw128(abase + off),
                      sdesc_mnmajor_sw128(bbase + st * 2048, kHalfBytes), idesc_kmn,
                      (term | st) ? 1u : 0u);
            }
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
    const int X = (warp - 1) >> 2;
    const int quarter = warp & 3;
    const int rr = 32 * quarter + lane;
    const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16);
    const uint32_t scol = tl + 128 * X;                 // S_X / P_X / OUT_X
    const uint32_t ocol = tl + 256 + 128 * X;           // O_X
    const RowId id = row_id(p, qb, X, rr);
    const bool valid = id.pos < p.Tq;
    const int64_t qpos = valid ? t_base + id.pos : qpos_max;
    const int64_t lim = p.causal ? qpos : p.n_tokens - 1;    // keys <= lim are seen
    const int64_t kst = row_kstart(p.kv_start, b);           // keys >= kst are seen
    bool ok = __all_sync(0xffffffffu, wait_or_abort(&bars[B_ROT], 0u, abort_flag, p.status));
    if (ok) {
      // q'_X (fp32, K order) -> fp16 A operand over Q_X
      tc::tc_fence_after();
      const uint32_t qdst = sbase + OFF_QA + X * kStage;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        tc::tmem_ld_x32(scol + 32 * c, x);
        tmem_ld_wait(x);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t h[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            h[e] = pack_half2(__uint_as_float(x[8 * q + 2 * e]), __uint_as_float(x[8 * q + 2 * e + 1]));
          sts128(qdst + sw_chunk(rr, 4 * c + q), make_uint4(h[0], h[1], h[2], h[3]));
        }
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cta(&bars[B_QP + X]);
    }
    float m = -INFINITY, l = 0.f;
    for (int j = 0; ok && j < ntiles; ++j) {
      ok = __all_sync(0xffffffffu, wait_or_abort(&bars[B_SFULL + X], (uint32_t)(j & 1),
                                                 abort_flag, p.status));
      if (!ok) break;
      tc::tc_fence_after();
      const int64_t k0 = (int64_t)j * kKeys;
      const bool need_mask = k0 + kKeys - 1 > lim || k0 < kst;
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
      // O_X += P_X(j-1) V^ is complete (S_X(j) was issued after it): rescale
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t x[32];
          tc::tmem_ld_x32(ocol + 32 * c, x);
          tmem_ld_wait(x);
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] = __float_as_uint(__uint_as_float(x[e]) * f);
          tc::tmem_st_x32(ocol + 32 * c, x);
        }
      }
      // pass 2: P = exp2(S - m) as fp16 pairs over the S columns (masked
      // scores are -inf: p = 0); l sums the fp16 values the PV MMA uses
      float l0 = 0.f, l1 = 0.f;
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
#pragma unroll
        for (int e = 0; e < 32; ++e) sum_f16x2(h[e], l0, l1);
        tc::tmem_st_x32(scol + 32 * hh, h);
      }
      l = l * f + (l0 + l1);
      tc::tmem_wait_st();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cta(&bars[B_PFULL + X]);
    }
    // O^_X = O_X / l (V order) -> fp16 hi / lo A operands (X = A: K stages,
    // X = B: V stages; every MMA of the loop is complete)
    if (ok)
      ok = __all_sync(0xffffffffu, wait_or_abort(&bars[B_ODONE], 0u, abort_flag, p.status));
    if (ok) {
      tc::tc_fence_after();
      const float il = l > 0.f ? 1.f / l : 0.f;
      const uint32_t ohi = sbase + (X == 0 ? OFF_K : OFF_V), olo = ohi + kStage;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        tc::tmem_ld_x32(ocol + 32 * c, x);
        tmem_ld_wait(x);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t h[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a = __uint_as_float(x[8 * q + 2 * e]) * il;
            const float bb = __uint_as_float(x[8 * q + 2 * e + 1]) * il;
            h[e] = pack_half2(a, bb);
            const __half2 hh = *reinterpret_cast<const __half2*>(&h[e]);
            lo[e] = pack_half2(a - __low2float(hh), bb - __high2float(hh));
          }
          sts128(ohi + sw_chunk(rr, 4 * c + q), make_uint4(h[0], h[1], h[2], h[3]));
          sts128(olo + sw_chunk(rr, 4 * c + q), make_uint4(lo[0], lo[1], lo[2], lo[3]));
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
      const int64_t h = kvh * p.g + (int64_t)chunk * p.hc + id.head;
      const int64_t base = b * p.os[0] + h * p.os[1] + (int64_t)id.pos * p.os[2];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t x[32];
        tc::tmem_ld_x32(scol + 32 * c, x);
        tmem_ld_wait(x);
        if (!valid) continue;
        if (p.o_vec) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) + base) + 4 * c;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t hv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float lo = __uint_as_float(x[8 * q + 2 * e]);
              const float hi = __uint_as_float(x[8 * q + 2 * e + 1]);
              if (p.o_dtype == TQ_F16) {
                hv[e] = pack_half2(lo, hi);
              } else {
                __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
                hv[e] = *reinterpret_cast<uint32_t*>(&v);
              }
            }
            dst[q] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
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
    // lane -> (key, part) as in tq_prefill_tc.cu (8 keys x 4 parts per warp,
    // conflict-free 16-byte stores); each thread takes its key row in both
    // pages
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
        // K^ of tile j + 1: both S MMAs of tile j - 1 have read this stage
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
      // V^ of tile j: both PV MMAs of tile j - 2 (or, for tile 0, the q'
      // MMAs, whose R_K sits in V stage 0) have read this stage
      const int s = j & 1;
      if (j >= 2)
        ok = wait_or_abort(&bars[B_VEMPTY + s], (uint32_t)(((j >> 1) - 1) & 1), abort_flag,
                           p.status);
      else if (j == 0)
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
    // R_V (MN-major B of OUT = O^ R_V): row i = R[v_coord(i)], fp16 hi over
    // q'_A and lo over q'_B, once the last S MMAs (which read q') are done
    if (ok) {
      const int jl = ntiles - 1;
      ok = __all_sync(0xffffffffu,
                      wait_or_abort(&bars[B_KEMPTY + (jl & 1)], (uint32_t)((jl >> 1) & 1),
                                    abort_flag, p.status));
    }
    if (ok) {
      for (int it = dt; it < kD * 16; it += kDecThreads) {
        const int i = it >> 4, c = it & 15;
        const float4* src = reinterpret_cast<const float4*>(p.rot + v_coord(i) * kD + 8 * c);
        const float4 a = __ldg(src), bq = __ldg(src + 1);
        const float v[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
        uint32_t h[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          h[e] = pack_half2(v[2 * e], v[2 * e + 1]);
          const __half2 hh = *reinterpret_cast<const __half2*>(&h[e]);
          lo[e] = pack_half2(v[2 * e] - __low2float(hh), v[2 * e + 1] - __high2float(hh));
        }
        sts128(sbase + OFF_QA + sw_chunk(i, c), make_uint4(h[0], h[1], h[2], h[3]));
        sts128(sbase + OFF_QB + sw_chunk(i, c), make_uint4(lo[0], lo[1], lo[2], lo[3]));
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

TcFn tc2_fn(int kb, int vb) {
#define TQ_PTC(K, V) if (kb == K && vb == V) return prefill_tc2_kernel<K, V>;
  TQ_PTC(4, 2) TQ_PTC(4, 4) TQ_PTC(3, 3) TQ_PTC(2, 2) TQ_PTC(3, 2) TQ_PTC(4, 3)
  TQ_PTC(2, 4) TQ_PTC(3, 4) TQ_PTC(2, 3) TQ_PTC(6, 4) TQ_PTC(5, 5) TQ_PTC(6, 6) TQ_PTC(5, 4)
#undef TQ_PTC
  return nullptr;
}

}  // namespace

int launch_prefill_tc2(const TcPrefillParams& base, int kb, int vb, int64_t B, int64_t Hq,
                       cudaStream_t st) {
  TcFn fn = tc2_fn(kb, vb);
  if (!fn) return 1;
  TcPrefillParams p = base;
  // two tiles of 128 rows: with hc >= 2 they split the heads, else the positions
  const int hct = p.hc >= 2 ? p.hc / 2 : 1;
  const int Pt = 128 / hct;
  p.pshift = 0;
  while ((1 << p.pshift) < Pt) ++p.pshift;
  p.pcta = p.hc >= 2 ? Pt : 256;
  p.tile_head_step = p.hc >= 2 ? hct : 0;
  p.tile_pos_step = p.hc >= 2 ? 0 : 128;
  p.nqb = (int)((p.Tq + p.pcta - 1) / p.pcta);
  // pair tables within 32 KB: 32 lane copies where they fit, else 16 / 8
  const int nk = 1 << (2 * kb), nv = 1 << (2 * vb);
  int rk = 32, rv = 32;
  while ((nk * rk + nv * rv) * 4 > (int)kLutMax) {
    if (nk * rk >= nv * rv) rk >>= 1; else rv >>= 1;
  }
  p.rk = rk;
  p.rv = rv;
  if (set_smem_attr((const void*)fn, SMEM_BYTES) != TQ_OK) return TQ_ERR_CUDA;
  dim3 grid((unsigned)p.nqb, (unsigned)(B * Hq / p.hc));
  fn<<<grid, kThreads, SMEM_BYTES, st>>>(p);
  return check_launch("tq_prefill_attn");
}

}  // namespace tq
