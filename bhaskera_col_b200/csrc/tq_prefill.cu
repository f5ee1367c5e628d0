// tq_prefill.cu — causal (or full) attention of a chunk of queries straight
// off the packed TurboQuant pages: the prefill attention of a layer.
//
// Replaces: HF attention (torch SDPA, causal, GQA repeat) over the
// dequantised K/V that TurboQuantKVCache.update returns during prefill
// (kv_cache.py:445-490 -> 483-488; engine.py:389).  The keys and values it
// attends are the reference's dequantised ones, x^ = n (c[idx] R): the MSE
// codes only (a QJL sketch, when the cache keeps one, refines decode scores
// and is not used here).
//
// Math, as in the decode kernel: <q, k_t> = n_t <q R^T, c_k[idx_t]> and
// sum_t p_t v_t = (sum_t p_t n_t c_v[idx_t]) R, so each CTA rotates its
// queries once, attends centroid values decoded from the codes, and
// un-rotates its output once.
//
// One CTA = 128 query rows of one KV head's GQA group: hc heads (the largest
// of 8, 4, 2, 1 dividing the group) x 128 / hc consecutive positions, 8 warps
// of 16 rows, so each decoded page serves hc heads.  Per 64-token page (one key tile): a bulk async copy brings the
// page into shared memory (double-buffered, mbarrier), all threads decode the
// K and V codes into fp16 tiles in coordinate order, then every warp runs
// S = Q' K^T and O += P' V with mma.sync m16n8k16 (fp16 in, fp32 accumulate)
// and an online softmax; P' = P * ||v|| folds the value norms in.
#include "tq_common.cuh"
#include "tq_internal.h"

#include <math.h>

namespace tq {
namespace {

constexpr int kPfWarps = 8;
constexpr int kPfThreads = 32 * kPfWarps;
constexpr float kLog2eP = 1.4426950408889634f;

struct PrefillParams {
  const uint8_t* pages;
  PageMap pm;
  int page_bytes, page_pitch, off_v, off_kn, off_vn;   // page geometry (make_geom)
  const __half* rot_h;          // R [D][D] fp16, row-major
  const float* kc;
  const float* vc;
  const void* q; int q_dtype; int64_t qs[4];     // (B, Hq, Tq, D)
  void* out; int o_dtype; int64_t os[4];
  int64_t Hq, Hkv, g, Tq, n_tokens;
  int hc;                       // query heads per CTA
  float scale;                  // softmax scale
  int causal;
  int nqb;                      // query blocks per head
  const int32_t* kv_start;      // [B] first attended key of each batch row, or NULL
  uint32_t* status;
};

template <int D, int KB, int VB>
struct Pf {
  static constexpr int KROW = D * KB / 8, VROW = D * VB / 8;
  static constexpr int LD = D + 8;                          // padded fp16 row (ldmatrix)
  static constexpr int OFF_R = 0;
  static constexpr int OFF_KS = OFF_R + D * LD * 2;
  static constexpr int OFF_VS = OFF_KS + 64 * LD * 2;
  static constexpr int OFF_NRM = OFF_VS + 64 * LD * 2;     // kn[64], vn[64] floats
  static constexpr int OFF_LUT = OFF_NRM + 512;            // K, V fp16 tables (256 each)
  static constexpr int OFF_BAR = OFF_LUT + 1024;
  static constexpr int OFF_STG = OFF_BAR + 128;            // 2 page stages (runtime size)
  static int smem(int page_pitch) { return OFF_STG + 2 * page_pitch; }
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}

// B fragments of two n-tiles (n0..n0+15) for k-chunk k0..k0+15 from a tile
// stored [n][k] (k contiguous, row stride ld halves).
__device__ __forceinline__ void frag_b_nk(uint32_t (&r)[4], const __half* base, int ld, int n0,
                                          int k0, int lane) {
  const int row = n0 + (lane & 7) + ((lane >> 4) << 3);
  const int col = k0 + (((lane >> 3) & 1) << 3);
  ldsm_x4(r, base + row * ld + col);
}
// Same from a tile stored [k][n] (n contiguous).
__device__ __forceinline__ void frag_b_kn(uint32_t (&r)[4], const __half* base, int ld, int n0,
                                          int k0, int lane) {
  const int row = k0 + (lane & 7) + (((lane >> 3) & 1) << 3);
  const int col = n0 + ((lane >> 4) << 3);
  ldsm_x4_t(r, base + row * ld + col);
}

template <int D, int KB, int VB>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_kernel(PrefillParams p) {
  using G = Pf<D, KB, VB>;
  constexpr int NC = D / 16;                  // 16-wide chunks of D
  constexpr int NT = D / 8;                   // 8-wide n-tiles of D
  extern __shared__ __align__(128) unsigned char smem[];
  __half* Rs = reinterpret_cast<__half*>(smem + G::OFF_R);
  __half* Ks = reinterpret_cast<__half*>(smem + G::OFF_KS);
  __half* Vs = reinterpret_cast<__half*>(smem + G::OFF_VS);
  float* kn = reinterpret_cast<float*>(smem + G::OFF_NRM);
  float* vn = kn + 64;
  __half* lutk = reinterpret_cast<__half*>(smem + G::OFF_LUT);
  __half* lutv = lutk + 256;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::OFF_BAR);
  const uint32_t PAGE = (uint32_t)p.page_bytes;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, tq = lane & 3;
  const int wph = kPfWarps / p.hc;                     // warps per head
  const int P = 16 * wph;                              // query positions per CTA
  const int qb = p.nqb - 1 - (int)blockIdx.x;          // long rows first
  const int nchunk = (int)(p.g / p.hc);
  const int64_t stream = (int64_t)blockIdx.y / nchunk;  // b * Hkv + kv head
  const int chunk = (int)((int64_t)blockIdx.y % nchunk);
  const int64_t b = stream / p.Hkv, kvh = stream % p.Hkv;
  const int64_t h = kvh * p.g + (int64_t)chunk * p.hc + warp / wph;   // this warp's head
  const int64_t t_base = p.n_tokens - p.Tq;            // position of query 0
  const int t0 = qb * P + (warp % wph) * 16;           // this warp's first query
  const int64_t qpos_max = t_base + tmin<int64_t>((int64_t)(qb + 1) * P, p.Tq) - 1;
  const int64_t kend = p.causal ? qpos_max + 1 : p.n_tokens;   // keys this CTA needs
  const int ntiles = (int)((kend + 63) / 64);
  int64_t kst = 0;                                     // first attended key (left padding)
  if (p.kv_start) {
    const int v = __ldg(p.kv_start + b);
    kst = v < 0 ? 0 : v;
  }

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_mbar_init();
  }
  // R (fp16) and the centroid tables
  for (int i = tid; i < D * D / 8; i += kPfThreads) {
    const int r = i / (D / 8), c8 = i % (D / 8);
    *reinterpret_cast<uint4*>(Rs + r * G::LD + c8 * 8) =
        __ldg(reinterpret_cast<const uint4*>(p.rot_h + r * D) + c8);
  }
  for (int i = tid; i < 256; i += kPfThreads) {
    lutk[i] = __float2half_rn(i < (1 << KB) ? __ldg(p.kc + i) : 0.f);
    lutv[i] = __float2half_rn(i < (1 << VB) ? __ldg(p.vc + i) : 0.f);
  }
  __syncthreads();
  // pool address of this stream's page pg (block table or contiguous)
  auto page_src = [&](int64_t pg) -> const uint8_t* {
    bool ok;
    const int64_t ps = page_slot(p.pm, stream, pg, ok);
    if (!ok) atomicOr(p.status, TQ_DEV_BAD_BLOCK);
    return p.pages + ps * (int64_t)PAGE;
  };
  if (tid == 0) {
    for (int i = 0; i < 2 && i < ntiles; ++i) {
      mbar_expect_tx(&full[i], PAGE);
      bulk_g2s(smem + G::OFF_STG + i * p.page_pitch, page_src(i), PAGE, &full[i]);
    }
  }

  // ---- queries: q' = (scale q) R^T as fp16 A fragments (log2e folded in) ----
  const bool active = t0 < p.Tq;
  uint32_t qf[NC][4];
  {
    const float sc = p.scale;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    const int64_t qbase = b * p.qs[0] + h * p.qs[1];
    const int r0 = t0 + gq, r1 = r0 + 8;
    auto ld2 = [&](int r, int c) -> uint32_t {
      if (r >= p.Tq) return 0u;
      const int64_t o = qbase + (int64_t)r * p.qs[2] + (int64_t)c * p.qs[3];
      return pack_half2(sc * load_elem(p.q, p.q_dtype, o), sc * load_elem(p.q, p.q_dtype, o + p.qs[3]));
    };
#pragma unroll
    for (int kc = 0; kc < NC; ++kc) {
      uint32_t a[4];
      a[0] = active ? ld2(r0, 16 * kc + 2 * tq) : 0u;
      a[1] = active ? ld2(r1, 16 * kc + 2 * tq) : 0u;
      a[2] = active ? ld2(r0, 16 * kc + 2 * tq + 8) : 0u;
      a[3] = active ? ld2(r1, 16 * kc + 2 * tq + 8) : 0u;
#pragma unroll
      for (int n = 0; n < NT; n += 2) {
        uint32_t bf[4];
        frag_b_nk(bf, Rs, G::LD, 8 * n, 16 * kc, lane);   // B[k][n] = R[n][k]
        mma_f16_16816(acc[n], a, bf[0], bf[1]);
        mma_f16_16816(acc[n + 1], a, bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int kc = 0; kc < NC; ++kc) {
      qf[kc][0] = pack_half2(acc[2 * kc][0] * kLog2eP, acc[2 * kc][1] * kLog2eP);
      qf[kc][1] = pack_half2(acc[2 * kc][2] * kLog2eP, acc[2 * kc][3] * kLog2eP);
      qf[kc][2] = pack_half2(acc[2 * kc + 1][0] * kLog2eP, acc[2 * kc + 1][1] * kLog2eP);
      qf[kc][3] = pack_half2(acc[2 * kc + 1][2] * kLog2eP, acc[2 * kc + 1][3] * kLog2eP);
    }
  }

  float O[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) O[n][0] = O[n][1] = O[n][2] = O[n][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int64_t qp0 = t_base + t0 + gq, qp1 = qp0 + 8;           // query positions
  const int64_t warp_kend = p.causal ? tmin<int64_t>(t_base + t0 + 16, p.n_tokens) : p.n_tokens;

  int kt = 0;
  for (; kt < ntiles; ++kt) {
    const int st = kt & 1;
    // every thread observes the copy; the block agrees on a timeout
    const bool ok = mbar_wait_bounded(&full[st], (uint32_t)((kt >> 1) & 1));
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicOr(p.status, TQ_DEV_WAIT_TIMEOUT);
      break;
    }
    const uint8_t* pg = smem + G::OFF_STG + st * p.page_pitch;
    // ---- decode K and V codes into fp16 tiles (coordinate order) ----------
    {
      // K: thread -> (token, quad); quad t of a row lists, for each chunk j,
      // coordinates 16j+2t, 16j+2t+1, 16j+2t+8, 16j+2t+9
      const int tok = tid >> 2, qd = tid & 3;
      constexpr int QB = (D / 4) * KB;                 // bits per quad
      const uint8_t* row = pg + tok * G::KROW;
      const int bit0 = qd * QB;
#pragma unroll
      for (int e = 0; e < D / 4; ++e) {
        const int bo = bit0 + e * KB;
        const uint32_t w = *reinterpret_cast<const uint32_t*>(row + ((bo >> 5) << 2));
        uint32_t code;
        if ((bo & 31) + KB <= 32) {
          code = (w >> (bo & 31)) & ((1u << KB) - 1u);
        } else {
          const uint32_t w2 = *reinterpret_cast<const uint32_t*>(row + ((bo >> 5) << 2) + 4);
          code = __funnelshift_r(w, w2, bo & 31) & ((1u << KB) - 1u);
        }
        const int j = e >> 2, r = e & 3;
        const int coord = 16 * j + 2 * qd + (r & 1) + ((r >> 1) << 3);
        Ks[tok * G::LD + coord] = lutk[code];
      }
      // V: thread -> (token, two octets); octet o lists coordinates o, o+8, ...
      constexpr int OB = (D / 8) * VB;                 // bits per octet
      const uint8_t* vrow = pg + p.off_v + tok * G::VROW;
#pragma unroll
      for (int oo = 0; oo < 2; ++oo) {
        const int oct = 2 * qd + oo;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          const int bo = oct * OB + c * VB;
          const uint32_t w = *reinterpret_cast<const uint32_t*>(vrow + ((bo >> 5) << 2));
          uint32_t code;
          if ((bo & 31) + VB <= 32) {
            code = (w >> (bo & 31)) & ((1u << VB) - 1u);
          } else {
            const uint32_t w2 = *reinterpret_cast<const uint32_t*>(vrow + ((bo >> 5) << 2) + 4);
            code = __funnelshift_r(w, w2, bo & 31) & ((1u << VB) - 1u);
          }
          Vs[tok * G::LD + oct + 8 * c] = lutv[code];
        }
      }
      if (tid < 64) {
        const int64_t key = (int64_t)kt * 64 + tid;
        const bool kok = key < kend;
        kn[tid] = kok ? __half2float(reinterpret_cast<const __half*>(pg + p.off_kn)[tid]) : 0.f;
        vn[tid] = kok ? __half2float(reinterpret_cast<const __half*>(pg + p.off_vn)[tid]) : 0.f;
      }
    }
    __syncthreads();
    // the stage is decoded: refill it with page kt + 2
    if (tid == 0 && kt + 2 < ntiles) {
      mbar_expect_tx(&full[st], PAGE);
      bulk_g2s(smem + G::OFF_STG + st * p.page_pitch, page_src(kt + 2), PAGE,
               &full[st]);
    }

    const int64_t k0 = (int64_t)kt * 64;
    if (active && k0 < warp_kend) {
      // ---- S = Q' K^T (16 x 64) -------------------------------------------
      float s[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < NC; ++kc) {
#pragma unroll
        for (int n = 0; n < 8; n += 2) {
          uint32_t bf[4];
          frag_b_nk(bf, Ks, G::LD, 8 * n, 16 * kc, lane);
          mma_f16_16816(s[n], qf[kc], bf[0], bf[1]);
          mma_f16_16816(s[n + 1], qf[kc], bf[2], bf[3]);
        }
      }
      // norms, causal mask, running max
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int kl = 8 * n + 2 * tq + c;
          const int64_t key = k0 + kl;
          const float nk = kn[kl];
          float v0 = s[n][c] * nk, v1 = s[n][2 + c] * nk;
          const bool lim0 = key < p.n_tokens && key >= kst && (!p.causal || key <= qp0);
          const bool lim1 = key < p.n_tokens && key >= kst && (!p.causal || key <= qp1);
          v0 = lim0 ? v0 : -INFINITY;
          v1 = lim1 ? v1 : -INFINITY;
          s[n][c] = v0;
          s[n][2 + c] = v1;
          mx0 = fmaxf(mx0, v0);
          mx1 = fmaxf(mx1, v1);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      if (mx0 > m0) {
        const float c = fast_exp2(m0 - mx0);
        l0 *= c;
#pragma unroll
        for (int n = 0; n < NT; ++n) { O[n][0] *= c; O[n][1] *= c; }
        m0 = mx0;
      }
      if (mx1 > m1) {
        const float c = fast_exp2(m1 - mx1);
        l1 *= c;
#pragma unroll
        for (int n = 0; n < NT; ++n) { O[n][2] *= c; O[n][3] *= c; }
        m1 = mx1;
      }
      const float b0 = m0 == -INFINITY ? 0.f : m0, b1 = m1 == -INFINITY ? 0.f : m1;
      // ---- P' = P * ||v|| as A fragments; O += P' V ----------------------
      uint32_t pa[4][4];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int kl = 8 * n + 2 * tq;
        const float p00 = fast_exp2(s[n][0] - b0), p01 = fast_exp2(s[n][1] - b0);
        const float p10 = fast_exp2(s[n][2] - b1), p11 = fast_exp2(s[n][3] - b1);
        l0 += p00 + p01;
        l1 += p10 + p11;
        const float w0 = vn[kl], w1 = vn[kl + 1];
        pa[n >> 1][(n & 1) * 2 + 0] = pack_half2(p00 * w0, p01 * w1);
        pa[n >> 1][(n & 1) * 2 + 1] = pack_half2(p10 * w0, p11 * w1);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          uint32_t bf[4];
          frag_b_kn(bf, Vs, G::LD, 8 * n, 16 * kk, lane);
          mma_f16_16816(O[n], a, bf[0], bf[1]);
          mma_f16_16816(O[n + 1], a, bf[2], bf[3]);
        }
      }
    }
    __syncthreads();   // the tiles are rewritten by the next decode
  }
  // after a timeout, never leave with a copy still writing shared memory:
  // tiles kt and kt + 1 may still be in flight
  if (tid == 0 && kt < ntiles) {
    for (int i = kt; i < tmin(kt + 2, ntiles); ++i)
      mbar_wait_bounded(&full[i & 1], (uint32_t)((i >> 1) & 1), 16u);
  }

  // ---- O = (O' / l) R, stored -----------------------------------------------
  if (active) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
    float acc[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < NC; ++kc) {
      uint32_t a[4];
      a[0] = pack_half2(O[2 * kc][0] * i0, O[2 * kc][1] * i0);
      a[1] = pack_half2(O[2 * kc][2] * i1, O[2 * kc][3] * i1);
      a[2] = pack_half2(O[2 * kc + 1][0] * i0, O[2 * kc + 1][1] * i0);
      a[3] = pack_half2(O[2 * kc + 1][2] * i1, O[2 * kc + 1][3] * i1);
#pragma unroll
      for (int n = 0; n < NT; n += 2) {
        uint32_t bf[4];
        frag_b_kn(bf, Rs, G::LD, 8 * n, 16 * kc, lane);   // B[k][n] = R[k][n]
        mma_f16_16816(acc[n], a, bf[0], bf[1]);
        mma_f16_16816(acc[n + 1], a, bf[2], bf[3]);
      }
    }
    const int r0 = t0 + gq, r1 = r0 + 8;
    const int64_t obase = b * p.os[0] + h * p.os[1];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int c = 8 * n + 2 * tq;
      if (r0 < p.Tq) {
        const int64_t o = obase + (int64_t)r0 * p.os[2] + (int64_t)c * p.os[3];
        store_elem(p.out, p.o_dtype, o, acc[n][0]);
        store_elem(p.out, p.o_dtype, o + p.os[3], acc[n][1]);
      }
      if (r1 < p.Tq) {
        const int64_t o = obase + (int64_t)r1 * p.os[2] + (int64_t)c * p.os[3];
        store_elem(p.out, p.o_dtype, o, acc[n][2]);
        store_elem(p.out, p.o_dtype, o + p.os[3], acc[n][3]);
      }
    }
  }
}

using PfFn = void (*)(PrefillParams);

template <int D>
PfFn pf_fn(int kb, int vb) {
#define TQ_PF(K, V) if (kb == K && vb == V) return prefill_kernel<D, K, V>;
  TQ_PF(4, 2) TQ_PF(3, 3) TQ_PF(2, 2) TQ_PF(4, 4) TQ_PF(6, 4) TQ_PF(5, 5) TQ_PF(6, 6)
  TQ_PF(8, 8) TQ_PF(3, 2) TQ_PF(4, 3)
#undef TQ_PF
  return nullptr;
}

}  // namespace

bool prefill_supported(int D, int kb, int vb) {
  if (D == 128) return pf_fn<128>(kb, vb) != nullptr;
  if (D == 64) return pf_fn<64>(kb, vb) != nullptr;
  return false;
}

int launch_prefill(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                   const tq_prefill_args* a, uint32_t* status, cudaStream_t st) {
  if (a->engine != 1) {
    const int rc = launch_prefill_tc(G, t, c, a, status, st);
    if (rc != 1) return rc;
  }
  PrefillParams p;
  const PageGeom g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  p.pages = c->pages;
  p.pm = page_map(c);
  p.page_bytes = g.page_bytes;
  p.page_pitch = (g.page_bytes + 127) & ~127;
  p.off_v = g.off_v;
  p.off_kn = g.off_kn;
  p.off_vn = g.off_vn;
  p.rot_h = reinterpret_cast<const __half*>(t->rot_f16);
  p.kc = t->k_centroids;
  p.vc = t->v_centroids;
  p.q = a->q->data; p.q_dtype = a->q->dtype;
  p.out = a->out->data; p.o_dtype = a->out->dtype;
  for (int i = 0; i < 4; ++i) { p.qs[i] = a->q->stride[i]; p.os[i] = a->out->stride[i]; }
  p.Hq = a->q->shape[1];
  p.Hkv = c->streams / a->q->shape[0];
  p.g = a->q->shape[1] / p.Hkv;
  p.hc = p.g % 8 == 0 ? 8 : p.g % 4 == 0 ? 4 : p.g % 2 == 0 ? 2 : 1;
  p.Tq = a->q->shape[2];
  p.n_tokens = a->n_tokens;
  p.scale = a->scale;
  p.causal = a->causal;
  p.kv_start = a->kv_start;
  p.nqb = (int)((p.Tq + 16 * (kPfWarps / p.hc) - 1) / (16 * (kPfWarps / p.hc)));
  p.status = status;
  if (p.Tq == 0) return TQ_OK;
  PfFn fn = G->head_dim == 128 ? pf_fn<128>(G->key_bits, G->value_bits)
                               : pf_fn<64>(G->key_bits, G->value_bits);
  const int smem = G->head_dim == 128 ? Pf<128, 4, 4>::smem(p.page_pitch)
                                      : Pf<64, 4, 4>::smem(p.page_pitch);
  if (!fn) {
    set_error("tq_prefill_attn: no kernel for head_dim %d, key_bits %d, value_bits %d",
              G->head_dim, G->key_bits, G->value_bits);
    return TQ_ERR_INVALID;
  }
  if (set_smem_attr((const void*)fn, smem) != TQ_OK) return TQ_ERR_CUDA;
  dim3 grid((unsigned)p.nqb, (unsigned)(a->q->shape[0] * p.Hq / p.hc));
  fn<<<grid, kPfThreads, smem, st>>>(p);
  return check_launch("tq_prefill_attn");
}

}  // namespace tq
