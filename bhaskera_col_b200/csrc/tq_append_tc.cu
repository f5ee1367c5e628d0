// tq_append_tc.cu — tensor-core append for head_dim 128, with or without
// the QJL sketch.
//
// Same result as append_kernel (kv_cache.py:382-398: fp32 norm of x,
// u = x / max(n, 1e-8), y = u R^T, codes = bucketize(y), fp16 norm; with QJL
// also the signs of z = S r for the residual r = y - c[code] and gamma =
// ||x|| ||r||) with both contractions on tcgen05 tensor cores:
//   * x (bf16) tiles of 128 consecutive tokens of one stream are loaded
//     exactly by TMA (128-byte swizzle, two 64-column halves);
//   * R = R_hi + R_mid + R_lo, three bf16 terms (24 significant bits), so
//     x R^T is the sum of three exact bf16 x bf16 products accumulated in fp32
//     in tensor memory (codes differ from an fp32 matmul only where y sits
//     within rounding of a boundary);
//   * the rows of each R term are permuted into the packed order of the row
//     (K quad order / V octet order), so TMEM column p holds the coordinate
//     stored at position p and every thread packs consecutive positions;
//   * the norm is ||x|| in fp32, summed from the bf16 tile in shared memory;
//   * QJL: the epilogue writes r (fp32, from the same thread's y) into tensor
//     memory as bf16 r_hi + r_lo (16 significant bits) and the MMA warp forms
//     z = r_hi S^T + r_lo S^T with S in bf16 (exact: the library's S is drawn
//     in bf16), A from tensor memory; z column q is the sketch coordinate at
//     K position q, so each thread packs one QJL word;
//   * one warp issues TMA, one warp issues the MMAs (M = N = 128, K = 16;
//     24 per tile, + 16 for the sketch) into one of two TMEM accumulators;
//     kSplit epilogue warps per TMEM lane quarter (2, or 4 with the sketch)
//     each take 128 / kSplit positions of 32 vectors.
//
// Bucketize, almost all on the fp32 pipe (the integer pipe issues at half
// the rate and bounded the first versions).  With w = 0.4 x the smallest
// boundary gap and cells c = 0..2L centred at (c - L) w, L = ceil(span / w) + 3:
//   u    = sat(y * inv / (2 L w) + 0.5)        (FFMA.SAT: clamps, NaN -> 0)
//   cell = round(2 L u)                        (FFMA against 2^23: the float's
//                                               low bits hold the integer)
//   {nbK, base, c[base], c[base + 1]} = lut[cell]  (one 16-byte load)
//   s    = sat((y * inv K + nbK) * K)          (= [y * inv > b] exactly:
//                                               nbK = -b K, K = 2^100, or -inf
//                                               when the cell's window
//                                               [c - L - 1, c - L + 1] w holds
//                                               no boundary; it holds <= 1.
//                                               The second scaling lifts every
//                                               nonzero difference, denormal
//                                               v included, to >= 2^51)
//   code = base + s = #{boundaries < v}        (torch.bucketize, right=False)
// Codes are packed by exact float arithmetic: acc = 2^23 + sum code_k 2^(BITS k)
// over runs of <= 23 bits, whose low float bits are the packed field.  The
// 16-byte table entries also carry c[base] and c[base + 1], the residual's
// centroid, and are replicated for 8 lanes (a 16-byte load serves 8 lanes per
// shared-memory phase, so a warp's lookups are conflict-free).  Tables that
// do not fit use a binary search instead.
//
// Every wait is bounded (mbar_wait_bounded); on expiry the kernel sets
// TQ_DEV_WAIT_TIMEOUT in a device status word (tq_device_status), drains its
// own copies and MMAs, frees its tensor memory and returns.
#include "tq_common.cuh"
#include "tq_internal.h"
#include "tq_tc.cuh"

#include <mutex>

namespace tq {
namespace {

constexpr int kD = 128;
constexpr int kM = 128;                    // vectors (tokens of one stream) per tile
constexpr int kHalf = kM * 64 * 2;         // 16 KB: 128 rows x 64 bf16, 128-byte swizzle
constexpr int kABytes = 2 * kHalf;         // one x tile
constexpr int kBBytes = 6 * kHalf;         // 3 terms of R x 2 K-halves
constexpr int kSBytes = 2 * kHalf;         // S (bf16) x 2 K-halves
constexpr float kCmpScale = 1.2676506e30f; // K = 2^100

// Epilogue shape.  Without the sketch: two warps per TMEM lane quarter, 64
// positions each, 8-byte lookup entries {-b K, base} replicated for 16 lanes
// (an 8-byte load serves 16 lanes per shared-memory phase).  With it: four
// warps per quarter, one K quad (32 positions, one QJL word) each, 16-byte
// entries that also carry c[base] and c[base + 1], replicated for 8 lanes.
// Either way a cell is 128 bytes of table.
template <bool QJL>
struct Epi {
  static constexpr int kSplit = QJL ? 4 : 2;       // epilogue warps per TMEM lane quarter
  static constexpr int kCW = kD / kSplit;          // positions per epilogue thread
  static constexpr int kEpiWarps = 4 * kSplit;
  static constexpr int kThreads = 32 * (2 + kEpiWarps);   // warp 0 TMA, warp 1 MMA, then epilogue
  static constexpr int kEntry = QJL ? 16 : 8;      // bytes per lookup entry
  static constexpr int kRep = 128 / kEntry;        // replicas per cell
};
constexpr int kCellShift = 7;                      // log2(bytes per cell)
// tensor memory: two 128-column fp32 accumulators of y; with the QJL sketch
// also the residual as a bf16 A operand (hi, lo: 64 columns each) and the
// 128-column fp32 accumulator of z = r S^T
constexpr uint32_t kColResHi = 256, kColResLo = 320, kColZ = 384;

template <bool QJL>
struct TcSmem {
  static constexpr int STAGES = QJL ? 2 : 3;
  static constexpr int OFF_B = 0;
  static constexpr int OFF_S = OFF_B + kBBytes;                  // QJL only
  static constexpr int OFF_A = OFF_S + (QJL ? kSBytes : 0);
  static constexpr int OFF_BND = OFF_A + STAGES * kABytes;       // [256] boundaries
  static constexpr int kSplit = Epi<QJL>::kSplit;
  static constexpr int OFF_XN = OFF_BND + 256 * 4;               // [2][kSplit][kM] partial ||x||^2
  static constexpr int OFF_RN = OFF_XN + 2 * kSplit * kM * 4;    // [kSplit][kM] partial ||r||^2
  static constexpr int OFF_BAR = OFF_RN + (QJL ? kSplit * kM * 4 : 0);
  static constexpr int OFF_LUT = OFF_BAR + 256;                  // lane-replicated cell table
  static constexpr int BYTES = 227 * 1024;
  static constexpr int LUT_BYTES = BYTES - 1024 - OFF_LUT;       // 1 KB: slack to align the base
  static constexpr uint32_t TMEM_COLS = QJL ? 512 : 256;
  static_assert(LUT_BYTES >= 8 * 1024, "shared memory");
  static_assert(OFF_A % 1024 == 0 && OFF_S % 1024 == 0 && kABytes % 1024 == 0,
                "swizzled tiles need 1 KB alignment");
};

struct TcParams {
  const float* bnd;
  const float* cent;
  int nb;
  uint8_t* pages;
  PageMap pm;
  int page_bytes, row_bytes, sec_off, norm_off;
  int qjl_off, gamma_off;                  // QJL sign rows and ||k|| ||r|| (K with QJL)
  int64_t H, T, pos, ntiles, nblk;
};

__device__ uint32_t g_tc_status;           // TQ_DEV_WAIT_TIMEOUT when a wait expired

__device__ __forceinline__ void fail() { atomicOr(&g_tc_status, TQ_DEV_WAIT_TIMEOUT); }

// bar.sync on a named barrier with an AND-reduction of `pred`: every thread
// of the group gets the same answer.
__device__ __forceinline__ bool group_and(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(nthreads) : "memory");
  return r != 0;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// bf16x2 of (lo, hi) rounded to nearest, lo in the low half
__device__ __forceinline__ uint32_t bf16x2_rn(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// D (+)= A B with A in tensor memory (lanes = rows, two 16-bit elements per
// column) and B in shared memory.
__device__ __forceinline__ void umma_ts_bf16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// One tile = 128 consecutive tokens of one stream.  With QJL (keys only) the
// epilogue also writes the rotated residual r = y - c[code] into tensor
// memory as bf16 hi + lo terms, the MMA warp forms z = r S^T (S exact in
// bf16, rows and columns in K quad order), and the epilogue packs the signs
// of z and stores gamma = ||k|| ||r||.
template <int BITS, bool QJL>
__global__ void __launch_bounds__(Epi<QJL>::kThreads, 1)
append_tc_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                 const __grid_constant__ CUtensorMap smap, TcParams p, int b_row0) {
  using SM = TcSmem<QJL>;
  constexpr int kAStages = SM::STAGES;
  constexpr int kSplit = Epi<QJL>::kSplit, kCW = Epi<QJL>::kCW, kEpiWarps = Epi<QJL>::kEpiWarps;
  constexpr int kThreads = Epi<QJL>::kThreads, kRep = Epi<QJL>::kRep;
  static_assert(!QJL || kCW == 32, "the sketch packs one QJL word per epilogue thread");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  unsigned char* sm = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + SM::OFF_BAR);
  uint64_t* b_full = bars;                      // 1
  uint64_t* a_full = bars + 1;                  // kAStages
  uint64_t* a_empty = a_full + kAStages;        // kAStages
  uint64_t* acc_full = a_empty + kAStages;      // 2
  uint64_t* acc_empty = acc_full + 2;           // 2
  uint64_t* res_full = acc_empty + 2;           // 1: the residual is in tensor memory
  uint64_t* z_full = res_full + 1;              // 1: z = r S^T is complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(z_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(z_full + 2);
  float* lutpar = reinterpret_cast<float*>(z_full + 3);   // 4 floats
  float* bnd = reinterpret_cast<float*>(sm + SM::OFF_BND);
  float* xn = reinterpret_cast<float*>(sm + SM::OFF_XN);
  float* rn = reinterpret_cast<float*>(sm + SM::OFF_RN);
  static_assert(3 * kAStages * 8 + 6 * 8 + 8 + 8 + 16 <= 256, "barrier block");

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = p.nb;

  if (tid == 0) {
    mbar_init(b_full, 1);
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1 + kEpiWarps);    // MMA commit + every epilogue warp's x read
    }
    for (int a = 0; a < 2; ++a) { mbar_init(&acc_full[a], 1); mbar_init(&acc_empty[a], kEpiWarps); }
    mbar_init(res_full, kEpiWarps);
    mbar_init(z_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, SM::TMEM_COLS);
    tc::tmem_relinquish();
  }
  for (int i = tid; i < nb; i += kThreads) bnd[i] = p.bnd[i];
  __syncthreads();
  // lookup grid (see the file comment); entries {-b K, base} (with the
  // sketch also c[base], c[base + 1]), replicated for kRep lanes
  if (tid == 0) {
    float gap = 1.f;
    for (int i = 0; i + 1 < nb; ++i) gap = fminf(gap, bnd[i + 1] - bnd[i]);
    const float w = 0.4f * gap;
    const float span = fmaxf(fabsf(bnd[0]), fabsf(bnd[nb - 1]));
    const float L = ceilf(span / w) + 3.f;
    const float nc = 2.f * L + 1.f;
    const bool ok = w > 0.f && nc * 128.f <= (float)SM::LUT_BYTES && span < 1.f;
    lutpar[0] = 1.f / (2.f * L * w);          // u = sat(v * lutpar[0] + 0.5)
    lutpar[1] = 2.f * L;                       // cell = round(u * 2L)
    lutpar[2] = ok ? nc : 0.f;
    lutpar[3] = w;
  }
  __syncthreads();
  const int ncells = (int)lutpar[2];
  const bool use_lut = ncells > 0;
  {
    const float w = lutpar[3], L = 0.5f * lutpar[1];
    for (int i = tid; i < ncells * kRep; i += kThreads) {
      const int c = i / kRep, l = i % kRep;
      const float wl = ((float)c - L - 1.f) * w, wh = ((float)c - L + 1.f) * w;
      int base = 0, hi = nb;                 // #boundaries < wl
      while (base < hi) {
        const int mid = (base + hi) >> 1;
        if (bnd[mid] < wl) base = mid + 1; else hi = mid;
      }
      const float nbk = (base < nb && bnd[base] <= wh) ? -bnd[base] * kCmpScale : -INFINITY;
      if constexpr (QJL) {
        const float clo = __ldg(p.cent + base), chi = __ldg(p.cent + tmin(base + 1, nb));
        reinterpret_cast<float4*>(sm + SM::OFF_LUT)[c * kRep + l] =
            make_float4(nbk, (float)base, clo, chi);
      } else {
        reinterpret_cast<float2*>(sm + SM::OFF_LUT)[c * kRep + l] = make_float2(nbk, (float)base);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(b_full, kBBytes + (QJL ? kSBytes : 0));
      for (int sp = 0; sp < 3; ++sp)
        for (int kh = 0; kh < 2; ++kh)
          tc::tma_load_2d(sm + SM::OFF_B + (sp * 2 + kh) * kHalf, &bmap, kh * 64, b_row0 + sp * kD,
                          b_full);
      if constexpr (QJL)
        for (int kh = 0; kh < 2; ++kh)
          tc::tma_load_2d(sm + SM::OFF_S + kh * kHalf, &smap, kh * 64, 0, b_full);
      int it = 0, issued = 0;
      for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++it) {
        const int st = it % kAStages;
        if (it >= kAStages &&
            !mbar_wait_bounded(&a_empty[st], (uint32_t)(((it / kAStages) - 1) & 1))) {
          fail();
          *abort_flag = 1;
        }
        if (*abort_flag) break;
        const int64_t s = tile / p.nblk, tb = tile % p.nblk;
        const int b = (int)(s / p.H), h = (int)(s % p.H), t0 = (int)(tb * kM);
        unsigned char* dst = sm + SM::OFF_A + st * kABytes;
        mbar_expect_tx(&a_full[st], kABytes);
        tc::tma_load_4d(dst, &amap, 0, t0, h, b, &a_full[st]);
        tc::tma_load_4d(dst + kHalf, &amap, 64, t0, h, b, &a_full[st]);
        issued = it + 1;
      }
      // never leave with a copy still writing shared memory
      for (int i = tmax(0, issued - kAStages); i < issued; ++i)
        mbar_wait_bounded(&a_full[i % kAStages], (uint32_t)((i / kAStages) & 1), 16u);
      mbar_wait_bounded(b_full, 0u, 16u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(kM, kD);
      const bool ok = mbar_wait_bounded(b_full, 0u);
      if (!ok) { fail(); *abort_flag = 1; }
      int it = 0, issued = 0, zdone = 0;
      const uint32_t bbase = smem_u32(sm + SM::OFF_B);
      const uint32_t sbase = smem_u32(sm + SM::OFF_S);
      // z = r S^T of tile `zi`, once its residual is in tensor memory
      auto issue_z = [&](int zi) -> bool {
        if (*abort_flag || !mbar_wait_bounded(res_full, (uint32_t)(zi & 1))) return false;
        tc::tc_fence_after();
#pragma unroll
        for (int term = 0; term < 2; ++term)
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t bd = tc::sdesc_kmajor_sw128(sbase + (ks >> 2) * kHalf + (ks & 3) * 32);
            umma_ts_bf16(tmem + kColZ, tmem + (term ? kColResLo : kColResHi) + 8 * ks, bd, idesc,
                         (term | ks) ? 1u : 0u);
          }
        tc::umma_commit(z_full);
        return true;
      };
      for (int64_t tile = blockIdx.x; ok && tile < p.ntiles; tile += gridDim.x, ++it) {
        const int st = it % kAStages, ac = it & 1;
        if (*abort_flag ||
            !mbar_wait_bounded(&a_full[st], (uint32_t)((it / kAStages) & 1)) ||
            (it >= 2 && !mbar_wait_bounded(&acc_empty[ac], (uint32_t)(((it / 2) - 1) & 1)))) {
          fail();
          *abort_flag = 1;
          break;
        }
        tc::tc_fence_after();
        const uint32_t abase = smem_u32(sm + SM::OFF_A + st * kABytes);
        const uint32_t d = tmem + (uint32_t)(ac * kD);
#pragma unroll
        for (int kh = 0; kh < 2; ++kh)
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
#pragma unroll
            for (int sp = 0; sp < 3; ++sp) {
              // K step of 16 bf16 = 32 bytes inside the 128-byte swizzled rows
              const uint64_t ad = tc::sdesc_kmajor_sw128(abase + kh * kHalf + ks * 32);
              const uint64_t bd = tc::sdesc_kmajor_sw128(bbase + (sp * 2 + kh) * kHalf + ks * 32);
              tc::umma_bf16(d, ad, bd, idesc, (kh | ks | sp) ? 1u : 0u);
            }
        tc::umma_commit(&a_empty[st]);
        tc::umma_commit(&acc_full[ac]);
        issued = it + 1;
        if constexpr (QJL) {
          // the previous tile's sketch, behind this tile's rotation
          if (it >= 1) {
            if (!issue_z(it - 1)) { fail(); *abort_flag = 1; break; }
            zdone = it;
          }
        }
      }
      if constexpr (QJL) {
        if (!*abort_flag && zdone < issued) {
          if (issue_z(issued - 1)) zdone = issued;
          else { fail(); *abort_flag = 1; }
        }
      }
      // the last commit tracks every MMA issued before it
      if (QJL && zdone > 0)
        mbar_wait_bounded(z_full, (uint32_t)((zdone - 1) & 1), 16u);
      else if (issued > 0)
        mbar_wait_bounded(&acc_full[(issued - 1) & 1], (uint32_t)(((issued - 1) / 2) & 1), 16u);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;                 // TMEM lane quarter this warp may read
    const int part = ew >> 2;               // which kCW positions of the row
    const int r = q * 32 + lane;            // tile row = vector
    int it = 0;
    for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, ++it) {
      const int st = it % kAStages, ac = it & 1;
      // (1) ||x||^2 over this part's kCW coordinates, from the swizzled tile
      bool ok = !*abort_flag && mbar_wait_bounded(&a_full[st], (uint32_t)((it / kAStages) & 1));
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        const unsigned char* xa = sm + SM::OFF_A + st * kABytes;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int c = 0; c < kCW / 8; ++c) {
          const int chunk = part * (kCW / 8) + c;        // 16-byte chunk of the row
          const int half = chunk >> 3, c8 = chunk & 7;
          const uint4 u = *reinterpret_cast<const uint4*>(xa + half * kHalf + r * 128 +
                                                          ((c8 ^ (r & 7)) << 4));
          tc::sq_bf16x2(u.x, s0, s1);
          tc::sq_bf16x2(u.y, s2, s3);
          tc::sq_bf16x2(u.z, s0, s1);
          tc::sq_bf16x2(u.w, s2, s3);
        }
        xn[((it & 1) * kSplit + part) * kM + r] = (s0 + s1) + (s2 + s3);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cta(&a_empty[st]);
      }
      // (2) the rotated row from tensor memory
      uint32_t yb[kCW];
      bool ok2 = ok && mbar_wait_bounded(&acc_full[ac], (uint32_t)((it / 2) & 1));
      ok2 = __all_sync(0xffffffffu, ok2);
      if (ok2) {
        tc::tc_fence_after();
#pragma unroll
        for (int c = 0; c < kCW / 32; ++c)
          tc::tmem_ld_x32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ac * kD + part * kCW + c * 32),
                          *reinterpret_cast<uint32_t(*)[32]>(yb + c * 32));
        tc::tmem_wait_ld();
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cta(&acc_empty[ac]);
      }
      // (3) the lane quarter's kSplit warps agree to go on (named barrier 1 + q)
      if (!group_and(1 + q, 32 * kSplit, ok2)) {
        if (lane == 0) { fail(); *abort_flag = 1; }
        break;
      }
      float ss = 0.f;
#pragma unroll
      for (int h = 0; h < kSplit; ++h) ss += xn[((it & 1) * kSplit + h) * kM + r];
      const float n = sqrtf(ss);
      const float inv = 1.f / fmaxf(n, 1e-8f);

      constexpr int NW = kCW * BITS / 32;
      uint32_t words[NW];
#pragma unroll
      for (int x = 0; x < NW; ++x) words[x] = 0u;
      uint32_t res[QJL ? kCW / 2 : 1];       // residual pairs (bf16 hi terms)
      float rss = 0.f;                       // this part's ||r||^2
      // a run of codes packed at bit offset o, len bits, as the float
      // acc = 2^23 + field (fields never overlap, so adding inserts them)
      auto flush = [&](float acc, int o, int len) {
        const uint32_t bits = __float_as_uint(acc);
        const int wi = o >> 5, sh = o & 31;
        if (sh + len <= 32) {
          // for sh >= 8 the exponent bits of 2^23 shift out of the word
          words[wi] += sh >= 8 ? (bits << sh) : ((bits & ((1u << len) - 1u)) << sh);
        } else {
          const uint32_t g = bits & ((1u << len) - 1u);
          words[wi] += g << sh;
          words[wi + 1] += g >> (32 - sh);
        }
      };
      if (use_lut) {
        const uint32_t lane_off = smem_u32(sm + SM::OFF_LUT) +
                                  (uint32_t)((lane % kRep) * Epi<QJL>::kEntry) -
                                  (0x4B000000u << kCellShift);
        const float ca = inv * lutpar[0], cK = inv * kCmpScale, c2l = lutpar[1];
        float acc = 8388608.f;
        int gs = 0, gl = 0;                    // run start bit / length (compile-time)
        float rprev = 0.f;
#pragma unroll
        for (int j = 0; j < kCW; ++j) {
          const int bo = j * BITS;
          if (gl > 0 && (gl + BITS > 23 || (bo & 31) == 0)) {
            flush(acc, gs, gl);
            acc = 8388608.f;
            gs = bo;
            gl = 0;
          }
          const float y = __uint_as_float(yb[j]);
          const float u = __saturatef(fmaf(y, ca, 0.5f));
          const float tc = fmaf(u, c2l, 8388608.f);
          const uint32_t ea = (__float_as_uint(tc) << kCellShift) + lane_off;
          float4 e;
          if constexpr (QJL) {
            e = lds_f4(ea);
          } else {
            const float2 e2 = tc::lds_f2(ea);
            e = make_float4(e2.x, e2.y, 0.f, 0.f);
          }
          const float sgt = __saturatef(fmaf(y, cK, e.x) * kCmpScale);
          acc = fmaf(e.y + sgt, (float)(1u << gl), acc);
          gl += BITS;
          if constexpr (QJL) {
            // r = y / n - c[code]: code = base + sgt picks c[base] or c[base + 1]
            const float rj = y * inv - (sgt > 0.5f ? e.w : e.z);
            rss = fmaf(rj, rj, rss);
            if (j & 1) res[j >> 1] = bf16x2_rn(rprev, rj);
            rprev = rj;
            yb[j] = __float_as_uint(rj);
          }
        }
        flush(acc, gs, gl);
      } else {
        auto put = [&](int j, uint32_t code) {
          const int bo = j * BITS, wi = bo >> 5, sh = bo & 31;
          words[wi] += code << sh;
          if (sh + BITS > 32) words[wi + 1] += code >> (32 - sh);
        };
        float rprev = 0.f;
#pragma unroll
        for (int j = 0; j < kCW; ++j) {
          const float y = __uint_as_float(yb[j]);
          const int code = bucketize_lt(bnd, nb, y * inv);
          put(j, (uint32_t)code);
          if constexpr (QJL) {
            const float rj = y * inv - __ldg(p.cent + code);
            rss = fmaf(rj, rj, rss);
            if (j & 1) res[j >> 1] = bf16x2_rn(rprev, rj);
            rprev = rj;
            yb[j] = __float_as_uint(rj);
          }
        }
      }
      const int64_t s = tile / p.nblk, tb = tile % p.nblk;
      const int64_t t = tb * kM + r;
      bool pok = true;
      const int64_t tp = p.pos + t;
      const int64_t ps = t < p.T ? page_slot(p.pm, s, tp / kPageTokens, pok) : 0;
      if (!pok) atomicOr(&g_tc_status, TQ_DEV_BAD_BLOCK);
      uint8_t* page = p.pages + ps * (int64_t)p.page_bytes;
      const int slot = (int)(tp % kPageTokens);
      const bool store = t < p.T && pok;
      if (store) {
        uint8_t* row = page + p.sec_off + slot * p.row_bytes + part * (kCW * BITS / 8);
        // widest store that the part's byte offset (part * NW * 4) keeps aligned
        if constexpr (NW % 4 == 0) {
#pragma unroll
          for (int x = 0; x < NW / 4; ++x)
            reinterpret_cast<uint4*>(row)[x] =
                make_uint4(words[4 * x], words[4 * x + 1], words[4 * x + 2], words[4 * x + 3]);
        } else if constexpr (NW % 2 == 0) {
#pragma unroll
          for (int x = 0; x < NW / 2; ++x)
            reinterpret_cast<uint2*>(row)[x] = make_uint2(words[2 * x], words[2 * x + 1]);
        } else {
#pragma unroll
          for (int x = 0; x < NW; ++x) reinterpret_cast<uint32_t*>(row)[x] = words[x];
        }
        if (part == 0) reinterpret_cast<__half*>(page + p.norm_off)[slot] = __float2half_rn(n);
      }
      if constexpr (QJL) {
        // (4) the residual into tensor memory: hi terms, then lo = r - hi
        uint32_t lo[kCW / 2];
#pragma unroll
        for (int i = 0; i < kCW / 2; ++i) {
          const float h0 = __uint_as_float(res[i] << 16), h1 = __uint_as_float(res[i] & 0xFFFF0000u);
          lo[i] = bf16x2_rn(__uint_as_float(yb[2 * i]) - h0, __uint_as_float(yb[2 * i + 1]) - h1);
        }
        const uint32_t lrow = (uint32_t)(q * 32) << 16;
        tc::tmem_st_x16(tmem + lrow + kColResHi + (uint32_t)(part * (kCW / 2)),
                        *reinterpret_cast<uint32_t(*)[16]>(res));
        tc::tmem_st_x16(tmem + lrow + kColResLo + (uint32_t)(part * (kCW / 2)),
                        *reinterpret_cast<uint32_t(*)[16]>(lo));
        tc::tmem_wait_st();
        rn[part * kM + r] = rss;
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cta(res_full);
        // (5) the signs of z for this part's positions (one QJL word)
        bool ok3 = mbar_wait_bounded(z_full, (uint32_t)(it & 1));
        ok3 = __all_sync(0xffffffffu, ok3);
        if (!group_and(1 + q, 32 * kSplit, ok3)) {
          if (lane == 0) { fail(); *abort_flag = 1; }
          break;
        }
        tc::tc_fence_after();
        uint32_t zb[32];
        tc::tmem_ld_x32(tmem + lrow + kColZ + (uint32_t)(part * kCW), zb);
        tc::tmem_wait_ld();
        // position e of quad `part` -> bit (e & 1) * 16 + (e >> 1)
        uint32_t sw = 0u;
#pragma unroll
        for (int e = 0; e < 32; ++e)
          sw |= (__uint_as_float(zb[e]) >= 0.f ? 1u : 0u) << ((e & 1) * 16 + (e >> 1));
        float rs = 0.f;
#pragma unroll
        for (int h = 0; h < kSplit; ++h) rs += rn[h * kM + r];
        if (store) {
          reinterpret_cast<uint32_t*>(page + p.qjl_off + slot * (kD / 8))[part] = sw;
          if (part == 0)
            reinterpret_cast<__half*>(page + p.gamma_off)[slot] = __float2half_rn(n * sqrtf(rs));
        }
        // rn and the z columns are rewritten only after the next tile's
        // agreement barrier (3) and residual barrier, which every part of
        // this lane quarter reaches after these reads
        tc::tc_fence_before();
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, SM::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static std::once_flag once;
  static EncodeTiled fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(f);
    else
      cudaGetLastError();
  });
  return fn;
}

using TcFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, TcParams, int);

template <bool QJL>
TcFn tc_fn_q(int bits) {
  switch (bits) {
    case 1: return append_tc_kernel<1, QJL>;
    case 2: return append_tc_kernel<2, QJL>;
    case 3: return append_tc_kernel<3, QJL>;
    case 4: return append_tc_kernel<4, QJL>;
    case 5: return append_tc_kernel<5, QJL>;
    case 6: return append_tc_kernel<6, QJL>;
    case 7: return append_tc_kernel<7, QJL>;
    case 8: return append_tc_kernel<8, QJL>;
    default: return nullptr;
  }
}

TcFn tc_fn(int bits, bool qjl) { return qjl ? tc_fn_q<true>(bits) : tc_fn_q<false>(bits); }

bool tc_view_ok(const tq_tensor4* x) {
  if (x->dtype != TQ_BF16 || x->shape[3] != kD || x->stride[3] != 1) return false;
  if (reinterpret_cast<uintptr_t>(x->data) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (x->stride[i] <= 0 || (x->stride[i] * 2) % 16) return false;
  return true;
}

}  // namespace

bool append_tc_applies(const tq_geom* G, const tq_tables* t, const tq_tensor4* k,
                       const tq_tensor4* v) {
  if (G->head_dim != kD || !t->rot_bf16x3) return false;
  if (G->qjl && (!t->qjl_bf16 || reinterpret_cast<uintptr_t>(t->qjl_bf16) % 16)) return false;
  if (!tc_view_ok(k) || !tc_view_ok(v) || k->shape[2] < 32) return false;
  if (!tc_fn(G->key_bits, G->qjl != 0) || !tc_fn(G->value_bits, false)) return false;
  if (reinterpret_cast<uintptr_t>(t->rot_bf16x3) % 16) return false;
  return encoder() != nullptr;
}

// Returns TQ_OK when launched, 1 when this path does not apply (the caller
// then uses the CUDA-core kernel), or an error.
int launch_append_tc(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                     const tq_tensor4* k, const tq_tensor4* v, int64_t pos, cudaStream_t st) {
  if (!append_tc_applies(G, t, k, v)) return 1;
  EncodeTiled enc = encoder();
  const PageGeom g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  auto map2d = [&](CUtensorMap* m, const void* base, int rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kD * 2};
    const cuuint32_t box[2] = {64, kD};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
               es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  // R terms: [2 orders][3 terms][128 rows][128] bf16, rows in packed order;
  // S: [128][128] bf16, rows and columns in K quad order
  CUtensorMap bmap, smap;
  if (!map2d(&bmap, t->rot_bf16x3, 6 * kD)) return 1;
  if (!map2d(&smap, G->qjl ? (const void*)t->qjl_bf16 : (const void*)t->rot_bf16x3, kD)) return 1;
  const int64_t B = k->shape[0], H = k->shape[1], T = k->shape[2];
  const int64_t nblk = (T + kM - 1) / kM;
  CUtensorMap amap[2];
  for (int which = 0; which < 2; ++which) {
    const tq_tensor4* x = which == 0 ? k : v;
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
    const cuuint64_t strides[3] = {(cuuint64_t)x->stride[2] * 2, (cuuint64_t)x->stride[1] * 2,
                                   (cuuint64_t)x->stride[0] * 2};
    const cuuint32_t box[4] = {64, kM, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (enc(&amap[which], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, x->data, dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return 1;
  }
  TcFn fns[2] = {tc_fn(G->key_bits, G->qjl != 0), tc_fn(G->value_bits, false)};
  for (int which = 0; which < 2; ++which)
    if (set_smem_attr((const void*)fns[which], TcSmem<false>::BYTES) != TQ_OK) return TQ_ERR_CUDA;
  const int sms = device_sm_count();
  for (int which = 0; which < 2; ++which) {
    TcParams p;
    p.bnd = which == 0 ? t->k_boundaries : t->v_boundaries;
    p.cent = which == 0 ? t->k_centroids : t->v_centroids;
    p.nb = (1 << (which == 0 ? G->key_bits : G->value_bits)) - 1;
    p.pages = c->pages;
    p.pm = page_map(c);
    p.page_bytes = g.page_bytes;
    p.row_bytes = which == 0 ? g.krow : g.vrow;
    p.sec_off = which == 0 ? g.off_k : g.off_v;
    p.norm_off = which == 0 ? g.off_kn : g.off_vn;
    p.qjl_off = g.off_q;
    p.gamma_off = g.off_kr;
    p.H = H; p.T = T; p.pos = pos;
    p.nblk = nblk;
    p.ntiles = B * H * nblk;
    const int grid = (int)tmin<int64_t>(p.ntiles, (int64_t)sms);
    const int threads = (which == 0 && G->qjl) ? Epi<true>::kThreads : Epi<false>::kThreads;
    fns[which]<<<grid, threads, TcSmem<false>::BYTES, st>>>(amap[which], bmap, smap, p, which * 3 * kD);
    if (check_launch("tq_append (tensor-core)") != TQ_OK) return TQ_ERR_CUDA;
  }
  return TQ_OK;
}

uint32_t* device_status_word() {
  void* addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_tc_status) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return static_cast<uint32_t*>(addr);
}

int read_tc_status(uint32_t* out, cudaStream_t st) {
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, g_tc_status);
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, addr, sizeof(uint32_t), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(addr, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) {
    set_error("tq_device_status: %s", cudaGetErrorString(e));
    return TQ_ERR_CUDA;
  }
  return *out ? TQ_ERR_DEVICE : TQ_OK;
}

}  // namespace tq
