// tq_decode.cu — single-token GQA decode attention straight off the packed
// TurboQuant pages.
//
// Replaces: HF attention (torch SDPA with GQA repeat) over the dequantised
// K/V that TurboQuantKVCache.update returns (aditya25058/Bhaskera_col
// src/bhaskera/inference/kv_cache.py:483-488, 580-589; engine.py:389).
//
// Math.  With R the layer rotation and k_t = n_t (c[idx_t] R), the score is
//   <q, k_t> = n_t <q R^T, c[idx_t]>,
// so the query is rotated once (qprep_kernel) and keys are never
// un-rotated.  Likewise o = sum_t p_t n_t (c_v[idx_t] R) = (sum_t p_t n_t
// c_v[idx_t]) R: values are accumulated in the rotated basis and un-rotated
// once per head in merge_kernel.  The optional QJL term adds
// gamma_t * alpha * <S q_rot, sign_t>.
//
// Kernels per call:
//   qprep_kernel   q_rot, S q_rot -> fp16 fragments (scale * log2e folded in)
//   decode_kernel  persistent; each CTA owns a contiguous range of the
//                  flattened (stream, page) space, streams 64-token pages
//                  into shared memory with bulk async copies (no multicast),
//                  dequantises codes into mma.sync fragments through
//                  lane-replicated pair lookup tables, runs an online
//                  softmax, and writes one partial (m, l, O_rot) per
//                  (stream, head, CTA) it touches.
//   merge_kernel   combines the partials of each (stream, head), attends the
//                  full-precision window, un-rotates, writes the output.
#include "tq_common.cuh"
#include "tq_internal.h"

#include <math.h>

namespace tq {

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kStages = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -INFINITY;

struct DecodeParams {
  PageGeom g;
  const uint8_t* pages;
  int64_t pages_per_stream;
  int64_t S, Pv, T, Q;
  int nch, maxslot;
  const uint32_t* qf;    // [S][nch][8][D/2] half2
  const uint32_t* sqf;   // [S][nch][8][D/2] half2
  const float* kc;
  const float* vc;
  float* part_m;         // [S][nch*8][maxslot]
  float* part_l;
  float* part_o;         // [S][nch*8][maxslot][D]
  uint32_t* status;
};

// ---------------------------------------------------------------------------
// bit helpers (offsets become compile-time constants after unrolling)
// ---------------------------------------------------------------------------
template <int NW>
__device__ __forceinline__ uint32_t getbits(const uint32_t (&w)[NW], int o, int n) {
  const int wi = o >> 5, sh = o & 31;
  uint32_t v;
  if (sh + n <= 32 || wi + 1 >= NW) v = w[wi] >> sh;
  else v = __funnelshift_r(w[wi], w[wi + 1], sh);
  return v & ((1u << n) - 1u);
}

// Load NBITS bits starting at bit `bit_off` of a 4-byte aligned smem row.
template <int NBITS, bool ALIGNED>
__device__ __forceinline__ void load_bits(const uint8_t* row, int bit_off,
                                          uint32_t (&w)[(NBITS + 31) / 32]) {
  constexpr int NW = (NBITS + 31) / 32;
  const uint32_t* p = reinterpret_cast<const uint32_t*>(row) + (bit_off >> 5);
  if constexpr (ALIGNED) {
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

// +-1 half2 from the two sign bits at positions pe (low half) and po (high).
__device__ __forceinline__ uint32_t sign_pair(uint32_t w, int pe, int po) {
  if (po == pe + 16 && pe <= 15) return 0xBC00BC00u ^ ((w << (15 - pe)) & 0x80008000u);
  uint32_t e = (w >> pe) & 1u, o = (w >> po) & 1u;
  return 0xBC00BC00u ^ ((e << 15) | (o << 31));
}

template <int BITS>
struct Lut {
  // pair tables for BITS <= 4: (1 << 2B) entries x 32 lanes of half2;
  // single-code tables otherwise: (1 << B) halves.
  static constexpr bool kPair = 2 * BITS <= 8;
  static constexpr int kWords = kPair ? (1 << (2 * BITS)) * 32 : ((1 << BITS) + 1) / 2;
};

template <int BITS>
__device__ __forceinline__ void build_lut(uint32_t* lut, const float* cent) {
  if constexpr (Lut<BITS>::kPair) {
    constexpr int E = 1 << (2 * BITS);
    for (int i = threadIdx.x; i < E * 32; i += blockDim.x) {
      int e = i >> 5;
      lut[i] = pack_half2(cent[e & ((1 << BITS) - 1)], cent[e >> BITS]);
    }
  } else {
    __half* h = reinterpret_cast<__half*>(lut);
    for (int i = threadIdx.x; i < (1 << BITS); i += blockDim.x) h[i] = __float2half_rn(cent[i]);
  }
}

// half2 of the codes (c_lo, c_hi)
template <int BITS>
__device__ __forceinline__ uint32_t lut_pair(const uint32_t* lut, uint32_t c_lo, uint32_t c_hi,
                                             int lane) {
  if constexpr (Lut<BITS>::kPair) {
    return lut[(((c_hi << BITS) | c_lo) << 5) + lane];
  } else {
    const unsigned short* h = reinterpret_cast<const unsigned short*>(lut);
    return (uint32_t)h[c_lo] | ((uint32_t)h[c_hi] << 16);
  }
}

// ---------------------------------------------------------------------------
// decode kernel
// ---------------------------------------------------------------------------
template <int D, int KB, int VB, bool QJL>
struct DecSmem {
  static constexpr int kLutK = Lut<KB>::kWords;
  static constexpr int kLutV = Lut<VB>::kWords;
  static constexpr int kComb = kDecWarps * (16 + 8 * D);
};

template <int D, int KB, int VB, bool QJL>
__global__ void __launch_bounds__(kDecThreads)
decode_kernel(DecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
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
  using SM = DecSmem<D, KB, VB, QJL>;

  const PageGeom& g = p.g;
  const int pb = (g.page_bytes + 127) & ~127;
  uint8_t* stage_buf = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * pb);
  uint32_t* lutK = reinterpret_cast<uint32_t*>(full + kStages);
  uint32_t* lutV = lutK + SM::kLutK;
  float* comb = reinterpret_cast<float*>(lutV + SM::kLutV);
  __shared__ int s_abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int hc = blockIdx.y;

  const int64_t TP = p.S * p.Pv;
  const int64_t gp0 = (int64_t)blockIdx.x * p.Q;
  const int64_t gp1 = tmin<int64_t>(gp0 + p.Q, TP);
  const int npages = (int)tmax<int64_t>(0, gp1 - gp0);

  build_lut<KB>(lutK, p.kc);
  build_lut<VB>(lutV, p.vc);
  if (tid == 0) {
    s_abort = 0;
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int i) {
    const int64_t gp = gp0 + i;
    const int64_t s = gp / p.Pv, pg = gp % p.Pv;
    const uint8_t* src = p.pages + (s * p.pages_per_stream + pg) * (int64_t)g.page_bytes;
    uint64_t* bar = &full[i % kStages];
    mbar_expect_tx(bar, (uint32_t)g.page_bytes);
    bulk_g2s(stage_buf + (i % kStages) * pb, src, (uint32_t)g.page_bytes, bar);
  };
  if (tid == 0) {
    for (int i = 0; i < kStages && i < npages; ++i) issue(i);
  }

  // per-thread state
  uint32_t qf[NJ][2], sqf[NJ][2];
  float O[NJ][4];
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
  int64_t cur_s = -1;

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
      qf[j][0] = qb[8 * j + tq];
      qf[j][1] = qb[8 * j + tq + 4];
      if constexpr (QJL) {
        sqf[j][0] = sb[8 * j + tq];
        sqf[j][1] = sb[8 * j + tq + 4];
      }
    }
  };
  reset_state();

  for (int i = 0; i < npages; ++i) {
    const int64_t gp = gp0 + i;
    const int64_t s = gp / p.Pv, pg = gp % p.Pv;
    if (s != cur_s) { load_q(s); cur_s = s; }

    if (!mbar_wait_bounded(&full[i % kStages], (uint32_t)((i / kStages) & 1))) {
      atomicOr(p.status, TQ_DEV_WAIT_TIMEOUT);
      s_abort = 1;
    }
    const uint8_t* pgb = stage_buf + (i % kStages) * pb;
    const int64_t tok0 = pg * kPageTokens + warp * 16;

    if (tok0 < p.T) {
      // ---------------- scores: S^T tile (16 tokens x 8 heads) --------------
      const int r0 = warp * 16 + gq, r1 = r0 + 8;
      uint32_t wk0[KQW], wk1[KQW];
      load_bits<KQB, KQA>(pgb + g.off_k + r0 * g.krow, tq * KQB, wk0);
      load_bits<KQB, KQA>(pgb + g.off_k + r1 * g.krow, tq * KQB, wk1);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      float acc2[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t wq0[QQW], wq1[QQW];
      if constexpr (QJL) {
        load_bits<QQB, (QQB % 32) == 0>(pgb + g.off_q + r0 * g.qrow, tq * QQB, wq0);
        load_bits<QQB, (QQB % 32) == 0>(pgb + g.off_q + r1 * g.qrow, tq * QQB, wq1);
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        uint32_t a[4];
        const int e0 = 4 * j;   // quad entries 4j..4j+3
        a[0] = lut_pair<KB>(lutK, getbits(wk0, e0 * KB, KB), getbits(wk0, (e0 + 1) * KB, KB), lane);
        a[1] = lut_pair<KB>(lutK, getbits(wk1, e0 * KB, KB), getbits(wk1, (e0 + 1) * KB, KB), lane);
        a[2] = lut_pair<KB>(lutK, getbits(wk0, (e0 + 2) * KB, KB), getbits(wk0, (e0 + 3) * KB, KB), lane);
        a[3] = lut_pair<KB>(lutK, getbits(wk1, (e0 + 2) * KB, KB), getbits(wk1, (e0 + 3) * KB, KB), lane);
        mma_f16_16816(acc, a, qf[j][0], qf[j][1]);
        if constexpr (QJL) {
          uint32_t b[4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int pr = 2 * j + h;                 // pair index in quad
            const int ch = pr / SP, pin = pr % SP;
            const int pe = ch * 2 * SP + pin, po = pe + SP;
            const int wi = pe >> 5;
            b[2 * h + 0] = sign_pair(wq0[wi], pe & 31, po - (wi << 5));
            b[2 * h + 1] = sign_pair(wq1[wi], pe & 31, po - (wi << 5));
          }
          uint32_t aq[4] = {b[0], b[1], b[2], b[3]};
          mma_f16_16816(acc2, aq, sqf[j][0], sqf[j][1]);
        }
      }
      const __half* kn = reinterpret_cast<const __half*>(pgb + g.off_kn);
      const __half* vn = reinterpret_cast<const __half*>(pgb + g.off_vn);
      const bool ok0 = tok0 + gq < p.T, ok1 = tok0 + gq + 8 < p.T;
      float n0 = __half2float(kn[r0]), n1 = __half2float(kn[r1]);
      float s00 = acc[0] * n0, s01 = acc[1] * n0, s10 = acc[2] * n1, s11 = acc[3] * n1;
      if constexpr (QJL) {
        const __half* kr = reinterpret_cast<const __half*>(pgb + g.off_kr);
        float g0 = __half2float(kr[r0]), g1 = __half2float(kr[r1]);
        s00 = fmaf(acc2[0], g0, s00); s01 = fmaf(acc2[1], g0, s01);
        s10 = fmaf(acc2[2], g1, s10); s11 = fmaf(acc2[3], g1, s11);
      }
      if (!ok0) { s00 = kNegInf; s01 = kNegInf; }
      if (!ok1) { s10 = kNegInf; s11 = kNegInf; }

      // ---------------- online softmax (columns = heads 2tq, 2tq+1) ---------
      float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float b0s = mn0 == kNegInf ? 0.f : mn0, b1s = mn1 == kNegInf ? 0.f : mn1;
      const float c0 = fast_exp2(m0 - b0s), c1 = fast_exp2(m1 - b1s);
      const float p00 = fast_exp2(s00 - b0s), p01 = fast_exp2(s01 - b1s);
      const float p10 = fast_exp2(s10 - b0s), p11 = fast_exp2(s11 - b1s);
      l0 = fmaf(l0, c0, p00 + p10);
      l1 = fmaf(l1, c1, p01 + p11);
      m0 = mn0; m1 = mn1;
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        O[i2][0] *= c0; O[i2][1] *= c1; O[i2][2] *= c0; O[i2][3] *= c1;
      }

      // ---------------- P' = p * ||v|| -> B fragments -----------------------
      const float v0 = ok0 ? __half2float(vn[r0]) : 0.f;
      const float v1 = ok1 ? __half2float(vn[r1]) : 0.f;
      const uint32_t pb0 = movmatrix_trans(pack_half2(p00 * v0, p01 * v0));
      const uint32_t pb1 = movmatrix_trans(pack_half2(p10 * v1, p11 * v1));

      // ---------------- O^T += V^T P ----------------------------------------
      const int t0r = warp * 16 + 2 * tq;
      uint32_t wa[VOW], wb[VOW], wc[VOW], wd[VOW];
      load_bits<VOB, VOA>(pgb + g.off_v + (t0r + 0) * g.vrow, gq * VOB, wa);
      load_bits<VOB, VOA>(pgb + g.off_v + (t0r + 1) * g.vrow, gq * VOB, wb);
      load_bits<VOB, VOA>(pgb + g.off_v + (t0r + 8) * g.vrow, gq * VOB, wc);
      load_bits<VOB, VOA>(pgb + g.off_v + (t0r + 9) * g.vrow, gq * VOB, wd);
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        uint32_t a[4];
        const int c0p = (2 * i2) * VB, c1p = (2 * i2 + 1) * VB;
        a[0] = lut_pair<VB>(lutV, getbits(wa, c0p, VB), getbits(wb, c0p, VB), lane);
        a[1] = lut_pair<VB>(lutV, getbits(wa, c1p, VB), getbits(wb, c1p, VB), lane);
        a[2] = lut_pair<VB>(lutV, getbits(wc, c0p, VB), getbits(wd, c0p, VB), lane);
        a[3] = lut_pair<VB>(lutV, getbits(wc, c1p, VB), getbits(wd, c1p, VB), lane);
        mma_f16_16816(O[i2], a, pb0, pb1);
      }
    }

    // ---------------- segment end: combine warps, emit partial ---------------
    const bool seg_end = (pg == p.Pv - 1) || (i == npages - 1);
    if (seg_end) {
      float L0 = l0, L1 = l1;
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        L0 += __shfl_xor_sync(0xffffffffu, L0, o);
        L1 += __shfl_xor_sync(0xffffffffu, L1, o);
      }
      float* cm = comb + warp * (16 + 8 * D);
      float* cl = cm + 8;
      float* co = cm + 16;
      if (gq == 0) {
        cm[2 * tq] = m0; cm[2 * tq + 1] = m1;
        cl[2 * tq] = L0; cl[2 * tq + 1] = L1;
      }
#pragma unroll
      for (int i2 = 0; i2 < NJ; ++i2) {
        co[(2 * tq) * D + 16 * i2 + gq] = O[i2][0];
        co[(2 * tq + 1) * D + 16 * i2 + gq] = O[i2][1];
        co[(2 * tq) * D + 16 * i2 + gq + 8] = O[i2][2];
        co[(2 * tq + 1) * D + 16 * i2 + gq + 8] = O[i2][3];
      }
      __syncthreads();
      const int64_t first = (s * p.Pv) / p.Q;
      const int slot = (int)(blockIdx.x - first);
      for (int idx = tid; idx < 8 * D; idx += kDecThreads) {
        const int h = idx / D, d = idx % D;
        float M = kNegInf;
#pragma unroll
        for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, comb[w * (16 + 8 * D) + h]);
        float Lsum = 0.f, Osum = 0.f;
        if (M != kNegInf) {
#pragma unroll
          for (int w = 0; w < kDecWarps; ++w) {
            const float* cw = comb + w * (16 + 8 * D);
            const float wt = fast_exp2(cw[h] - M);
            Lsum = fmaf(wt, cw[8 + h], Lsum);
            Osum = fmaf(wt, cw[16 + h * D + d], Osum);
          }
        }
        const int64_t hrow = (s * p.nch + hc) * 8 + h;
        p.part_o[(hrow * p.maxslot + slot) * D + d] = Osum;
        if (d == 0) {
          p.part_m[hrow * p.maxslot + slot] = M;
          p.part_l[hrow * p.maxslot + slot] = Lsum;
        }
      }
      reset_state();
    }
    __syncthreads();
    if (s_abort) break;
    if (tid == 0 && i + kStages < npages) issue(i + kStages);
  }
  // Drain: make sure no bulk copy is still writing this CTA's shared memory.
  if (s_abort && tid == 0) {
    for (int i = 0; i < npages && i < kStages; ++i) {
      // bounded; a copy that never lands leaves the status flag set
      mbar_wait_bounded(&full[i], 0u, 1u << 16);
    }
  }
}

// ---------------------------------------------------------------------------
// query preparation: q_rot = q R^T, sq = S q_rot, scaled, packed to half2
// grid = (S, nch), 128 threads
// ---------------------------------------------------------------------------
struct QPrepParams {
  int D, g, Hkv, nch;
  const void* q; int q_dtype; int64_t q_stride[4];
  const float* R; const float* Sm;
  float scale_q, scale_s;
  uint32_t* qf; uint32_t* sqf;
};

__global__ void __launch_bounds__(128) qprep_kernel(QPrepParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int D = p.D;
  float* qs = reinterpret_cast<float*>(smem);   // [8][D]
  float* qr = qs + 8 * D;                        // [8][D]
  const int64_t s = blockIdx.x;
  const int hc = blockIdx.y;
  const int64_t b = s / p.Hkv, kvh = s % p.Hkv;
  for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) {
    const int hl = i / D, c = i % D;
    const int hg = hc * 8 + hl;
    float v = 0.f;
    if (hg < p.g) {
      const int64_t hq = kvh * p.g + hg;
      v = load_elem(p.q, p.q_dtype, b * p.q_stride[0] + hq * p.q_stride[1] + c * p.q_stride[3]);
    }
    qs[i] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) {
    const int hl = i / D, j = i % D;
    float acc = 0.f;
    for (int k = 0; k < D; ++k) acc = fmaf(qs[hl * D + k], __ldg(p.R + j * D + k), acc);
    qr[i] = acc;
  }
  __syncthreads();
  uint32_t* qo = p.qf + (s * p.nch + hc) * 8 * (D / 2);
  for (int i = threadIdx.x; i < 8 * (D / 2); i += blockDim.x) {
    const int hl = i / (D / 2), c2 = i % (D / 2);
    qo[i] = pack_half2(qr[hl * D + 2 * c2] * p.scale_q, qr[hl * D + 2 * c2 + 1] * p.scale_q);
  }
  if (p.Sm) {
    for (int i = threadIdx.x; i < 8 * D; i += blockDim.x) {
      const int hl = i / D, j = i % D;
      float acc = 0.f;
      for (int k = 0; k < D; ++k) acc = fmaf(qr[hl * D + k], __ldg(p.Sm + j * D + k), acc);
      qs[i] = acc;
    }
    __syncthreads();
    uint32_t* so = p.sqf + (s * p.nch + hc) * 8 * (D / 2);
    for (int i = threadIdx.x; i < 8 * (D / 2); i += blockDim.x) {
      const int hl = i / (D / 2), c2 = i % (D / 2);
      so[i] = pack_half2(qs[hl * D + 2 * c2] * p.scale_s, qs[hl * D + 2 * c2 + 1] * p.scale_s);
    }
  }
}

// ---------------------------------------------------------------------------
// merge: combine partials, add the window, un-rotate, store
// grid = (S, nch), 128 threads
// ---------------------------------------------------------------------------
struct MergeParams {
  int D, g, Hkv, nch, maxslot;
  int64_t Pv, Q;
  const float* part_m; const float* part_l; const float* part_o;
  const float* R;
  const void* q; int q_dtype; int64_t q_stride[4];
  const void* wk; const void* wv; int w_dtype; int64_t wk_stride[4], wv_stride[4]; int64_t W;
  float scale_log2;       // softmax scale * log2(e)
  void* out; int out_dtype; int64_t out_stride[4];
};

__global__ void __launch_bounds__(128) merge_kernel(MergeParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int D = p.D;
  float* orot = reinterpret_cast<float*>(smem);   // [D]
  float* qv = orot + D;                            // [D]
  float* ow = qv + D;                              // [D]
  float* sc = ow + D;                              // [W]
  __shared__ float s_red[32];
  __shared__ float s_stats[4];
  const int64_t s = blockIdx.x;
  const int hc = blockIdx.y;
  const int64_t b = s / p.Hkv, kvh = s % p.Hkv;
  const int tid = threadIdx.x;
  int nslot = 0;
  if (p.Pv > 0) {
    const int64_t first = (s * p.Pv) / p.Q, last = ((s + 1) * p.Pv - 1) / p.Q;
    nslot = (int)(last - first + 1);
  }
  for (int hl = 0; hl < 8 && hc * 8 + hl < p.g; ++hl) {
    const int64_t hq = kvh * p.g + hc * 8 + hl;
    const int64_t hrow = (s * p.nch + hc) * 8 + hl;
    // --- window scores (unrotated) -----------------------------------------
    float mw = -INFINITY;
    if (p.W > 0) {
      for (int c = tid; c < D; c += blockDim.x)
        qv[c] = load_elem(p.q, p.q_dtype, b * p.q_stride[0] + hq * p.q_stride[1] + c * p.q_stride[3]);
      __syncthreads();
      const int warp = tid >> 5, lane = tid & 31;
      for (int64_t t = warp; t < p.W; t += blockDim.x / 32) {
        float acc = 0.f;
        for (int c = lane; c < D; c += 32)
          acc = fmaf(qv[c], load_elem(p.wk, p.w_dtype, b * p.wk_stride[0] + kvh * p.wk_stride[1] +
                                                         t * p.wk_stride[2] + c * p.wk_stride[3]), acc);
        acc = warp_sum(acc);
        if (lane == 0) sc[t] = acc * p.scale_log2;
      }
      __syncthreads();
      float mloc = -INFINITY;
      for (int64_t t = tid; t < p.W; t += blockDim.x) mloc = fmaxf(mloc, sc[t]);
      for (int o = 16; o > 0; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
      if ((tid & 31) == 0) s_red[tid >> 5] = mloc;
      __syncthreads();
      if (tid == 0) {
        float m = -INFINITY;
        for (int w = 0; w < (int)(blockDim.x / 32); ++w) m = fmaxf(m, s_red[w]);
        s_stats[0] = m;
      }
      __syncthreads();
      mw = s_stats[0];
    }
    // --- global max ----------------------------------------------------------
    float M = mw;
    for (int k = 0; k < nslot; ++k) M = fmaxf(M, p.part_m[hrow * p.maxslot + k]);
    const float Ms = (M == -INFINITY) ? 0.f : M;
    // --- rotated partial combination ---------------------------------------
    float L = 0.f;
    for (int k = 0; k < nslot; ++k) {
      const float mk = p.part_m[hrow * p.maxslot + k];
      if (mk != -INFINITY) L = fmaf(exp2f(mk - Ms), p.part_l[hrow * p.maxslot + k], L);
    }
    for (int d = tid; d < D; d += blockDim.x) {
      float acc = 0.f;
      for (int k = 0; k < nslot; ++k) {
        const float mk = p.part_m[hrow * p.maxslot + k];
        if (mk != -INFINITY)
          acc = fmaf(exp2f(mk - Ms), p.part_o[(hrow * p.maxslot + k) * D + d], acc);
      }
      orot[d] = acc;
    }
    // --- window contribution (unrotated) -----------------------------------
    float lw = 0.f;
    for (int d = tid; d < D; d += blockDim.x) ow[d] = 0.f;
    __syncthreads();
    if (p.W > 0) {
      for (int64_t t = tid; t < p.W; t += blockDim.x) sc[t] = exp2f(sc[t] - Ms);
      __syncthreads();
      for (int64_t t = 0; t < p.W; ++t) lw += sc[t];
      for (int d = tid; d < D; d += blockDim.x) {
        float acc = 0.f;
        for (int64_t t = 0; t < p.W; ++t)
          acc = fmaf(sc[t], load_elem(p.wv, p.w_dtype, b * p.wv_stride[0] + kvh * p.wv_stride[1] +
                                                        t * p.wv_stride[2] + d * p.wv_stride[3]), acc);
        ow[d] = acc;
      }
      __syncthreads();
    }
    const float Ltot = L + lw;
    const float inv = Ltot > 0.f ? 1.f / Ltot : 0.f;
    for (int j = tid; j < D; j += blockDim.x) {
      float acc = 0.f;
      for (int d = 0; d < D; ++d) acc = fmaf(orot[d], __ldg(p.R + d * D + j), acc);
      store_elem(p.out, p.out_dtype,
                 b * p.out_stride[0] + hq * p.out_stride[1] + j * p.out_stride[3],
                 (acc + ow[j]) * inv);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

struct Plan {
  int D, g, nch, maxslot, ctas;
  int64_t S, Pv, T, Q;
  size_t off_qf, off_sqf, off_m, off_l, off_o, total;
};

using DecodeFn = void (*)(DecodeParams);

template <int D, int KB, int VB, bool QJL>
size_t dec_smem_bytes(int page_bytes) {
  using SM = DecSmem<D, KB, VB, QJL>;
  const size_t pb = (size_t)((page_bytes + 127) & ~127);
  return kStages * pb + kStages * 8 + (size_t)(SM::kLutK + SM::kLutV) * 4 + (size_t)SM::kComb * 4;
}

struct Variant {
  int D, kb, vb, qjl;
  DecodeFn fn;
  size_t (*smem)(int);
};

#define TQ_VARIANT(D_, KB_, VB_, Q_) \
  {D_, KB_, VB_, Q_, decode_kernel<D_, KB_, VB_, (Q_ != 0)>, dec_smem_bytes<D_, KB_, VB_, (Q_ != 0)>}
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

const Variant* find_variant(const tq_geom* g) {
  for (const Variant& v : kVariants)
    if (v.D == g->head_dim && v.kb == g->key_bits && v.vb == g->value_bits && v.qjl == (g->qjl != 0))
      return &v;
  return nullptr;
}

Plan make_plan(const tq_geom* G, const tq_cache* c, const tq_decode_args* a, int occ) {
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
  pl.Q = TP > 0 ? (TP + slots - 1) / slots : 1;
  pl.ctas = TP > 0 ? (int)((TP + pl.Q - 1) / pl.Q) : 0;
  pl.maxslot = pl.Pv > 0 ? (int)((pl.Pv + pl.Q - 1) / pl.Q + 1) : 1;
  size_t off = 256;
  const size_t heads = (size_t)pl.S * pl.nch * 8;
  pl.off_qf = off;  off += heads * (pl.D / 2) * 4;
  pl.off_sqf = off; off += heads * (pl.D / 2) * 4;
  off = (off + 255) & ~(size_t)255;
  pl.off_m = off;   off += heads * pl.maxslot * 4;
  pl.off_l = off;   off += heads * pl.maxslot * 4;
  off = (off + 255) & ~(size_t)255;
  pl.off_o = off;   off += heads * pl.maxslot * pl.D * 4;
  pl.total = (off + 255) & ~(size_t)255;
  return pl;
}

int occupancy_of(const Variant* v, size_t smem) {
  return occupancy((const void*)v->fn, kDecThreads, smem);
}

}  // namespace

size_t decode_workspace_bytes(const tq_geom* g, const tq_cache* c, const tq_decode_args* a) {
  const Variant* v = find_variant(g);
  if (!v) return 0;
  const PageGeom pg = make_geom(g->head_dim, g->key_bits, g->value_bits, g->qjl);
  const size_t smem = v->smem(pg.page_bytes);
  if (set_smem_attr((const void*)v->fn, smem) != TQ_OK) return 0;
  return make_plan(g, c, a, occupancy_of(v, smem)).total;
}

int launch_decode(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                  const tq_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t st) {
  const Variant* v = find_variant(G);
  if (!v) {
    set_error("tq_decode_attn: no kernel for head_dim=%d key_bits=%d value_bits=%d qjl=%d",
              G->head_dim, G->key_bits, G->value_bits, G->qjl);
    return TQ_ERR_INVALID;
  }
  const PageGeom pg = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  const size_t smem = v->smem(pg.page_bytes);
  if (set_smem_attr((const void*)v->fn, smem) != TQ_OK) return TQ_ERR_CUDA;
  const Plan pl = make_plan(G, c, a, occupancy_of(v, smem));
  if (ws == nullptr || ws_bytes < pl.total) {
    set_error("tq_decode_attn: workspace of %zu bytes needed, %zu given", pl.total, ws_bytes);
    return TQ_ERR_WORKSPACE;
  }
  uint8_t* w = static_cast<uint8_t*>(ws);
  const int64_t Hkv = c->streams / a->q->shape[0];
  const float alpha = sqrtf(3.14159265358979f / 2.f) / (float)pl.D;

  QPrepParams qp;
  qp.D = pl.D; qp.g = pl.g; qp.Hkv = (int)Hkv; qp.nch = pl.nch;
  qp.q = a->q->data; qp.q_dtype = a->q->dtype;
  for (int i = 0; i < 4; ++i) qp.q_stride[i] = a->q->stride[i];
  qp.R = t->rot; qp.Sm = G->qjl ? t->qjl : nullptr;
  qp.scale_q = a->scale * kLog2e;
  qp.scale_s = a->scale * kLog2e * alpha;
  qp.qf = reinterpret_cast<uint32_t*>(w + pl.off_qf);
  qp.sqf = reinterpret_cast<uint32_t*>(w + pl.off_sqf);
  const int phases = a->phases ? a->phases : (TQ_PHASE_QPREP | TQ_PHASE_DECODE | TQ_PHASE_MERGE);
  if (pl.S > 0 && (phases & TQ_PHASE_QPREP)) {
    qprep_kernel<<<dim3((unsigned)pl.S, pl.nch), 128, 2 * 8 * pl.D * 4, st>>>(qp);
    if (check_launch("tq_decode_attn/qprep") != TQ_OK) return TQ_ERR_CUDA;
  }

  DecodeParams dp;
  dp.g = pg;
  dp.pages = c->pages; dp.pages_per_stream = c->pages_per_stream;
  dp.S = pl.S; dp.Pv = pl.Pv; dp.T = pl.T; dp.Q = pl.Q;
  dp.nch = pl.nch; dp.maxslot = pl.maxslot;
  dp.qf = qp.qf; dp.sqf = qp.sqf;
  dp.kc = t->k_centroids; dp.vc = t->v_centroids;
  dp.part_m = reinterpret_cast<float*>(w + pl.off_m);
  dp.part_l = reinterpret_cast<float*>(w + pl.off_l);
  dp.part_o = reinterpret_cast<float*>(w + pl.off_o);
  dp.status = reinterpret_cast<uint32_t*>(w);
  if (pl.ctas > 0 && (phases & TQ_PHASE_DECODE)) {
    v->fn<<<dim3(pl.ctas, pl.nch), kDecThreads, smem, st>>>(dp);
    if (check_launch("tq_decode_attn/decode") != TQ_OK) return TQ_ERR_CUDA;
  }

  MergeParams mp;
  mp.D = pl.D; mp.g = pl.g; mp.Hkv = (int)Hkv; mp.nch = pl.nch; mp.maxslot = pl.maxslot;
  mp.Pv = pl.Pv; mp.Q = pl.Q;
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
  if (pl.S > 0 && (phases & TQ_PHASE_MERGE)) {
    const size_t msmem = (size_t)(3 * pl.D + (mp.W > 0 ? mp.W : 1)) * 4;
    if (set_smem_attr((const void*)merge_kernel, msmem) != TQ_OK) return TQ_ERR_CUDA;
    merge_kernel<<<dim3((unsigned)pl.S, pl.nch), 128, msmem, st>>>(mp);
    if (check_launch("tq_decode_attn/merge") != TQ_OK) return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

}  // namespace tq
