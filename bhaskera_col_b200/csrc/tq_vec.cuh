// tq_vec.cuh — per-vector append math shared by the append and decode-step
// kernels, so both write bit-identical pages.
//
// Follows _LayerKVStore._compress_chunk (aditya25058/Bhaskera_col
// src/bhaskera/inference/kv_cache.py:382-398): fp32 norm, u = x / max(n,
// 1e-8), y = u R^T, code = #{boundaries < y}, stored norm = fp16(n).
#pragma once

#include "tq_common.cuh"

namespace tq {

// One warp: u[0..D) = x / max(||x||, 1e-8) (x read with stride sd from
// base), returns ||x|| on every lane.
__device__ __forceinline__ float warp_normalize(const void* x, int dtype, int64_t base,
                                                int64_t sd, float* u, int D, int lane) {
  float ss = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float xv = load_elem(x, dtype, base + c * sd);
    u[c] = xv;
    ss = fmaf(xv, xv, ss);
  }
  ss = warp_sum(ss);
  const float n = sqrtf(ss);
  const float den = fmaxf(n, 1e-8f);
  __syncwarp();
  for (int c = lane; c < D; c += 32) u[c] = u[c] / den;
  return n;
}

// y_j = sum_i u[i] T[i][j] (T row-major, i ascending).
__device__ __forceinline__ float rot_coord(const float* u, const float* T, int j, int D) {
  float acc = 0.f;
  for (int i = 0; i < D; ++i) acc = fmaf(u[i], T[i * D + j], acc);
  return acc;
}

// acc[v] = sum_i x[v * ldx + i] T[i][j] for NV vectors at once (same per-vector
// summation order as rot_coord, so results are bit-identical); vectors with
// v >= nv are skipped.
template <int D, int NV>
__device__ __forceinline__ void rot_multi(const float* x, int ldx, int nv, const float* T, int j,
                                          float (&acc)[NV]) {
#pragma unroll
  for (int v = 0; v < NV; ++v) acc[v] = 0.f;
#pragma unroll 4
  for (int i = 0; i < D; ++i) {
    const float t = T[i * D + j];
#pragma unroll
    for (int v = 0; v < NV; ++v)
      if (v < nv) acc[v] = fmaf(x[v * ldx + i], t, acc[v]);
  }
}

// rot_multi with four coordinates of each vector per broadcast load (x rows
// 16-byte aligned, ldx a multiple of 4): the same per-vector summation order
// (i ascending, one fmaf per term), so the results are bit-identical.
template <int D, int NV>
__device__ __forceinline__ void rot_multi4(const float* x, int ldx, int nv, const float* T, int j,
                                           float (&acc)[NV]) {
  static_assert(D % 4 == 0, "head_dim");
#pragma unroll
  for (int v = 0; v < NV; ++v) acc[v] = 0.f;
#pragma unroll 2
  for (int i = 0; i < D; i += 4) {
    const float t0 = T[i * D + j], t1 = T[(i + 1) * D + j];
    const float t2 = T[(i + 2) * D + j], t3 = T[(i + 3) * D + j];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if (v < nv) {
        const float4 xv = *reinterpret_cast<const float4*>(x + v * ldx + i);
        acc[v] = fmaf(xv.x, t0, acc[v]);
        acc[v] = fmaf(xv.y, t1, acc[v]);
        acc[v] = fmaf(xv.z, t2, acc[v]);
        acc[v] = fmaf(xv.w, t3, acc[v]);
      }
    }
  }
}

// acc[v] = sum_i x[row[v] * D + i] T[i][j] for the first N vectors, i
// ascending with one fmaf per term (rot_coord's order, so each result is
// bit-identical to it).  N is a compile-time count and every load is
// unconditional, so the loads of an unrolled block issue together instead
// of one latency at a time.
template <int D, int N, int NA>
__device__ __forceinline__ void rot_rows_n(const float* x, const int (&row)[NA], const float* T,
                                           int j, float (&acc)[NA]) {
  const float* xp[N];
#pragma unroll
  for (int v = 0; v < N; ++v) {
    acc[v] = 0.f;
    xp[v] = x + row[v] * D;
  }
  // x rows are 16-byte aligned shared-memory rows: four coordinates of each
  // vector come in one broadcast load (one wavefront per vector and four
  // steps instead of four), the FMA order per vector unchanged
  static_assert(D % 4 == 0, "head_dim");
#pragma unroll 2
  for (int i = 0; i < D; i += 4) {
    const float t0 = T[i * D + j], t1 = T[(i + 1) * D + j];
    const float t2 = T[(i + 2) * D + j], t3 = T[(i + 3) * D + j];
#pragma unroll
    for (int v = 0; v < N; ++v) {
      const float4 xv = *reinterpret_cast<const float4*>(xp[v] + i);
      acc[v] = fmaf(xv.x, t0, acc[v]);
      acc[v] = fmaf(xv.y, t1, acc[v]);
      acc[v] = fmaf(xv.z, t2, acc[v]);
      acc[v] = fmaf(xv.w, t3, acc[v]);
    }
  }
}

// rot_rows_n for nv (<= NA, uniform across the warp) vectors at rows row[v].
template <int D, int NA>
__device__ __forceinline__ void rot_rows(const float* x, const int (&row)[NA], int nv,
                                         const float* T, int j, float (&acc)[NA]) {
  static_assert(NA >= 1 && NA <= 5, "vectors per thread");
  switch (nv) {
    case 1: rot_rows_n<D, 1, NA>(x, row, T, j, acc); break;
    case 2: if constexpr (NA >= 2) rot_rows_n<D, 2, NA>(x, row, T, j, acc); break;
    case 3: if constexpr (NA >= 3) rot_rows_n<D, 3, NA>(x, row, T, j, acc); break;
    case 4: if constexpr (NA >= 4) rot_rows_n<D, 4, NA>(x, row, T, j, acc); break;
    case 5: if constexpr (NA >= 5) rot_rows_n<D, 5, NA>(x, row, T, j, acc); break;
    default: break;
  }
}

// Word w of a packed row: LSB-first stream of `bits`-bit codes taken in the
// order ord[position] -> coordinate.
__device__ __forceinline__ uint32_t pack_word(const uint8_t* code, const int16_t* ord, int bits,
                                              int w, int D) {
  const int b0 = 32 * w;
  const int n0 = b0 / bits, n1 = (b0 + 31) / bits;
  uint64_t acc = 0;
  for (int n = n0; n <= n1 && n < D; ++n) {
    const uint64_t cv = code[ord[n]];
    const int rel = n * bits - b0;
    acc |= rel >= 0 ? (cv << rel) : (cv >> (-rel));
  }
  return (uint32_t)acc;
}

// Word w of a QJL row from 0/1 signs; qinv[bit] -> coordinate.
__device__ __forceinline__ uint32_t pack_qjl_word(const uint8_t* qb, const int16_t* qinv, int w) {
  uint32_t word = 0;
  for (int bit = 0; bit < 32; ++bit) word |= (uint32_t)qb[qinv[32 * w + bit]] << bit;
  return word;
}

// pack_word by one warp: lane l holds bit 32w + l of the row (bit b of the
// code at position n, 32w + l = n * bits + b), and the ballot is the word.
// Same bits as pack_word; every lane gets the word.
__device__ __forceinline__ uint32_t ballot_word(const uint8_t* code, const int16_t* ord,
                                                int bits, int w, int D, int lane) {
  const int bit = 32 * w + lane;
  const int n = bit / bits, b = bit - n * bits;
  const bool v = n < D && ((code[ord[n]] >> b) & 1);
  return __ballot_sync(0xffffffffu, v);
}

// Position -> coordinate tables of the K (quad) and V (octet) row orders and
// the QJL bit -> coordinate table.
__device__ __forceinline__ void build_orders(int16_t* ordk, int16_t* ordv, int16_t* qinv, int D,
                                             int tid, int nthreads) {
  for (int c = tid; c < D; c += nthreads) {
    const int kp = k_pos_of(c, D);
    if (ordk) ordk[kp] = (int16_t)c;
    if (qinv) qinv[qjl_bit_of(kp, D)] = (int16_t)c;
    if (ordv) ordv[v_pos_of(c, D)] = (int16_t)c;
  }
}

}  // namespace tq
