// tq_append.cu — bucketize, fused append (norm -> rotate -> quantize -> pack
// -> QJL sketch) and dequantisation for the packed TurboQuant cache.
//
// Reference math (aditya25058/Bhaskera_col):
//   norm / normalise / rotate / bucketize / store  kv_cache.py:378-398
//   dequantise + un-rotate + rescale               kv_cache.py:422-439
#include "tq_common.cuh"
#include "tq_internal.h"
#include "tq_vec.cuh"

namespace tq {

// ---------------------------------------------------------------------------
// Bit-exact quantiser on an already rotated fp32 tensor.
// ---------------------------------------------------------------------------
__global__ void quantize_rotated_kernel(const float* __restrict__ y, int64_t n,
                                        const float* __restrict__ bnd, int nb,
                                        int16_t* __restrict__ codes) {
  __shared__ float sb[256];
  for (int i = threadIdx.x; i < nb; i += blockDim.x) sb[i] = bnd[i];
  __syncthreads();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    codes[i] = (int16_t)bucketize_lt(sb, nb, y[i]);
  }
}

// ---------------------------------------------------------------------------
// Fused append (CUDA cores, fp32).  One CTA processes tiles of kAppendVT
// vectors of one tensor (blockIdx.y: 0 = K, 1 = V); R^T (and S^T for K with
// QJL) stay resident in shared memory across tiles.  The tables take most of
// an SM's shared memory, so one CTA of 16 warps per SM shares them (4 warps
// and 16-vector tiles ran at 73 GB/s); the rotations read four coordinates
// of a vector per broadcast load.
// ---------------------------------------------------------------------------
constexpr int kVT = 16;                  // dequantisation tile (tokens)
constexpr int kAppendVT = 64;            // append tile (vectors)
constexpr int kAppendThreads = 512;

struct AppendParams {
  PageGeom g;
  const float* cent[2];
  const float* bnd[2];
  const float* RT;      // R^T row-major
  const float* ST;      // S^T row-major (QJL)
  int vt;               // vectors per tile (<= kAppendVT)
  uint8_t* pages;
  PageMap pm;
  uint32_t* status;     // TQ_DEV_BAD_BLOCK on a block-table entry outside the pool
  const void* x[2];
  int dtype[2];
  int64_t stride[2][4];
  int64_t B, H, T;
  int64_t pos;
};

template <int D>
__global__ void __launch_bounds__(kAppendThreads)
append_kernel(AppendParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int GR = kAppendThreads / D;  // vector groups
  constexpr int NV = (kAppendVT + GR - 1) / GR; // vectors per thread
  const int which = blockIdx.y;           // 0: K, 1: V
  const PageGeom& g = p.g;
  const int bits = which == 0 ? g.kb : g.vb;
  const bool qjl = (which == 0) && g.qjl;
  const int nb = (1 << bits) - 1;

  float* RT = reinterpret_cast<float*>(smem);                 // [D][D]
  float* ST = RT + D * D;                                     // [D][D] (qjl)
  float* u = ST + (qjl ? D * D : 0);                          // [kAppendVT][D]
  float* yv = u + kAppendVT * D;                              // [kAppendVT][D]
  float* cb = yv + kAppendVT * D;                             // [256]
  float* bb = cb + 256;                                       // [256]
  float* nrm = bb + 256;                                      // [kAppendVT]
  float* gam = nrm + kAppendVT;                               // [kAppendVT]
  uint8_t* code = reinterpret_cast<uint8_t*>(gam + kAppendVT);      // [kAppendVT][D]
  uint8_t* qb = code + kAppendVT * D;                         // [kAppendVT][D]
  int16_t* ord = reinterpret_cast<int16_t*>(qb + kAppendVT * D);    // [D] pos -> coord
  int16_t* qinv = ord + D;                                    // [D] bit -> coord

  const int tid = threadIdx.x;
  // R^T (and S^T) as given, all 16-byte copies in flight at once
  stage_async(RT, p.RT, D * D * 4, tid, blockDim.x);
  if (qjl) stage_async(ST, p.ST, D * D * 4, tid, blockDim.x);
  cp_async_wait_all();
  for (int i = tid; i < (1 << bits); i += blockDim.x) cb[i] = p.cent[which][i];
  for (int i = tid; i < nb; i += blockDim.x) bb[i] = p.bnd[which][i];
  if (which == 0) build_orders(ord, nullptr, qinv, D, tid, blockDim.x);
  else build_orders(nullptr, ord, nullptr, D, tid, blockDim.x);
  __syncthreads();

  const int64_t nvec = p.B * p.H * p.T;
  const int vt = p.vt;
  const int64_t ntiles = (nvec + vt - 1) / vt;
  const int lane = tid & 31, warp = tid >> 5;
  const int rowbytes = which == 0 ? g.krow : g.vrow;
  const int sec = which == 0 ? g.off_k : g.off_v;
  const int nsec = which == 0 ? g.off_kn : g.off_vn;

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t v0 = tile * vt;
    const int nv = (int)tmin<int64_t>(vt, nvec - v0);

    // -- load + norm + normalise (one warp per vector) ----------------------
    for (int v = warp; v < nv; v += kAppendThreads / 32) {
      int64_t gv = v0 + v;
      int64_t t = gv % p.T, bh = gv / p.T, h = bh % p.H, b = bh / p.H;
      const int64_t* st = p.stride[which];
      const int64_t base = b * st[0] + h * st[1] + t * st[2];
      const float n = warp_normalize(p.x[which], p.dtype[which], base, st[3], u + v * D, D, lane);
      if (lane == 0) nrm[v] = n;
    }
    __syncthreads();

    // -- rotate: y[v][j] = sum_i u[v][i] R[j][i], all of a thread's vectors --
    {
      const int j = tid % D, grp = tid / D;
      const int mine = (grp < GR && nv > grp) ? (nv - grp + GR - 1) / GR : 0;
      float acc[NV];
      rot_multi4<D, NV>(u + grp * D, GR * D, mine, RT, j, acc);
#pragma unroll
      for (int k = 0; k < NV; ++k) {
        if (k < mine) {
          const int v = grp + k * GR;
          yv[v * D + j] = acc[k];
          code[v * D + j] = (uint8_t)bucketize_lt(bb, nb, acc[k]);
        }
      }
    }
    __syncthreads();

    // -- QJL: residual r = y - c[idx] (reuse u), z = S r, gamma = n ||r|| ----
    if (qjl) {
      for (int i = tid; i < nv * D; i += blockDim.x) u[i] = yv[i] - cb[code[i]];
      __syncthreads();
      {
        const int j = tid % D, grp = tid / D;
        const int mine = (grp < GR && nv > grp) ? (nv - grp + GR - 1) / GR : 0;
        float acc[NV];
        rot_multi4<D, NV>(u + grp * D, GR * D, mine, ST, j, acc);
#pragma unroll
        for (int k = 0; k < NV; ++k)
          if (k < mine) qb[(grp + k * GR) * D + j] = acc[k] >= 0.f ? 1 : 0;
      }
      for (int v = warp; v < nv; v += kAppendThreads / 32) {
        float ss = 0.f;
        for (int c = lane; c < D; c += 32) ss = fmaf(u[v * D + c], u[v * D + c], ss);
        ss = warp_sum(ss);
        if (lane == 0) gam[v] = nrm[v] * sqrtf(ss);
      }
      __syncthreads();
    }

    // -- pack rows and store ------------------------------------------------
    const int words = rowbytes / 4;
    for (int i = tid; i < nv * words; i += blockDim.x) {
      const int v = i / words, w = i % words;
      const int64_t gv = v0 + v;
      const int64_t t = gv % p.T + p.pos, s = gv / p.T;
      bool ok;
      const int64_t ps = page_slot(p.pm, s, t / kPageTokens, ok);
      if (!ok) { atomicOr(p.status, TQ_DEV_BAD_BLOCK); continue; }
      uint8_t* page = p.pages + ps * (int64_t)g.page_bytes;
      const int slot = (int)(t % kPageTokens);
      reinterpret_cast<uint32_t*>(page + sec + slot * rowbytes)[w] =
          pack_word(code + v * D, ord, bits, w, D);
    }
    if (qjl) {
      const int qwords = D / 32;
      for (int i = tid; i < nv * qwords; i += blockDim.x) {
        const int v = i / qwords, w = i % qwords;
        const int64_t gv = v0 + v;
        const int64_t t = gv % p.T + p.pos, s = gv / p.T;
        bool ok;
        const int64_t ps = page_slot(p.pm, s, t / kPageTokens, ok);
        if (!ok) continue;
        uint8_t* page = p.pages + ps * (int64_t)g.page_bytes;
        const int slot = (int)(t % kPageTokens);
        reinterpret_cast<uint32_t*>(page + g.off_q + slot * g.qrow)[w] =
            pack_qjl_word(qb + v * D, qinv, w);
      }
    }
    for (int v = tid; v < nv; v += blockDim.x) {
      const int64_t gv = v0 + v;
      const int64_t t = gv % p.T + p.pos, s = gv / p.T;
      bool ok;
      const int64_t ps = page_slot(p.pm, s, t / kPageTokens, ok);
      if (!ok) continue;
      uint8_t* page = p.pages + ps * (int64_t)g.page_bytes;
      const int slot = (int)(t % kPageTokens);
      reinterpret_cast<__half*>(page + nsec)[slot] = __float2half_rn(nrm[v]);
      if (qjl) reinterpret_cast<__half*>(page + g.off_kr)[slot] = __float2half_rn(gam[v]);
    }
    __syncthreads();
  }
}

size_t append_smem_bytes(int D, bool qjl) {
  size_t f = (size_t)D * D * (qjl ? 2 : 1) + 2 * kAppendVT * D + 512 + 2 * kAppendVT;
  return f * 4 + 2 * kAppendVT * D + 2 * D * sizeof(int16_t) + 16;
}

// ---------------------------------------------------------------------------
// Dequantisation: x = (c[idx] R) * norm for tokens [t0, t1) of every stream.
// grid = (ceil((t1-t0)/kVT), streams, 2)
// ---------------------------------------------------------------------------
struct DequantParams {
  PageGeom g;
  const float* cent[2];
  const float* R;
  const uint8_t* pages;
  PageMap pm;
  uint32_t* status;
  int64_t H;
  int64_t t0, t1;
  void* out[2];
  int dtype[2];
  int64_t stride[2][4];
};

__global__ void __launch_bounds__(128) dequant_kernel(DequantParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int which = blockIdx.z;
  if (p.out[which] == nullptr) return;
  const PageGeom& g = p.g;
  const int D = g.D;
  const int bits = which == 0 ? g.kb : g.vb;
  float* cv = reinterpret_cast<float*>(smem);   // [kVT][D]
  float* nr = cv + kVT * D;                     // [kVT]
  const int64_t s = blockIdx.y;
  const int64_t tt0 = p.t0 + (int64_t)blockIdx.x * kVT;
  const int nv = (int)tmin<int64_t>(kVT, p.t1 - tt0);
  const int rowbytes = which == 0 ? g.krow : g.vrow;
  const int sec = which == 0 ? g.off_k : g.off_v;
  const int nsec = which == 0 ? g.off_kn : g.off_vn;
  const float* cent = p.cent[which];
  for (int i = threadIdx.x; i < nv * D; i += blockDim.x) {
    const int v = i / D, c = i % D;
    const int64_t t = tt0 + v;
    bool ok;
    const int64_t ps = page_slot(p.pm, s, t / kPageTokens, ok);
    if (!ok) atomicOr(p.status, TQ_DEV_BAD_BLOCK);
    const uint8_t* page = p.pages + ps * (int64_t)g.page_bytes;
    const uint8_t* row = page + sec + (t % kPageTokens) * rowbytes;
    const int pos = which == 0 ? k_pos_of(c, D) : v_pos_of(c, D);
    const int bo = pos * bits;
    uint32_t w = 0;
    for (int k = 0; k < bits; ++k) {
      int bb = bo + k;
      w |= (uint32_t)((row[bb >> 3] >> (bb & 7)) & 1) << k;
    }
    cv[v * D + c] = cent[w];
    if (c == 0) nr[v] = __half2float(reinterpret_cast<const __half*>(page + nsec)[t % kPageTokens]);
  }
  __syncthreads();
  const int64_t b = s / p.H, h = s % p.H;
  const int64_t* st = p.stride[which];
  for (int i = threadIdx.x; i < nv * D; i += blockDim.x) {
    const int v = i / D, j = i % D;
    float acc = 0.f;
    for (int k = 0; k < D; ++k) acc = fmaf(cv[v * D + k], __ldg(p.R + k * D + j), acc);
    const int64_t t = tt0 + v - p.t0;
    store_elem(p.out[which], p.dtype[which], b * st[0] + h * st[1] + t * st[2] + j * st[3],
               acc * nr[v]);
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
int launch_quantize_rotated(const float* y, int64_t n, const float* b, int nb,
                            int16_t* codes, cudaStream_t st) {
  if (n == 0) return TQ_OK;
  int blocks = (int)tmin<int64_t>((n + 255) / 256, 148 * 8);
  quantize_rotated_kernel<<<blocks, 256, 0, st>>>(y, n, b, nb, codes);
  return check_launch("tq_quantize_rotated");
}

int launch_append(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                  const tq_tensor4* k, const tq_tensor4* v, int64_t pos,
                  cudaStream_t st) {
  AppendParams p;
  p.g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  p.cent[0] = t->k_centroids; p.cent[1] = t->v_centroids;
  p.bnd[0] = t->k_boundaries; p.bnd[1] = t->v_boundaries;
  p.RT = t->rot_t; p.ST = t->qjl_t;
  p.pages = c->pages; p.pm = page_map(c); p.status = device_status_word();
  p.x[0] = k->data; p.x[1] = v->data;
  p.dtype[0] = k->dtype; p.dtype[1] = v->dtype;
  for (int i = 0; i < 4; ++i) { p.stride[0][i] = k->stride[i]; p.stride[1][i] = v->stride[i]; }
  p.B = k->shape[0]; p.H = k->shape[1]; p.T = k->shape[2];
  p.pos = pos;
  const int64_t nvec = p.B * p.H * p.T;
  if (nvec == 0) return TQ_OK;
  if (const int rc = launch_append_tc(G, t, c, k, v, pos, st); rc != 1) return rc;
  const size_t smem = append_smem_bytes(p.g.D, p.g.qjl != 0);
  void (*fn)(AppendParams) = p.g.D == 32 ? append_kernel<32>
                           : p.g.D == 64 ? append_kernel<64>
                           : p.g.D == 96 ? append_kernel<96> : append_kernel<128>;
  if (set_smem_attr((const void*)fn, smem) != TQ_OK) return TQ_ERR_CUDA;
  const int sms = device_sm_count();
  const int occ = tmax(1, occupancy((const void*)fn, kAppendThreads, smem));
  // small appends (decode steps): few vectors per CTA so the grid fills the
  // GPU; large appends: full tiles, persistent CTAs
  const int64_t want = (nvec + (int64_t)sms * occ - 1) / ((int64_t)sms * occ);
  p.vt = (int)tmax<int64_t>(1, tmin<int64_t>(kAppendVT, 2 * want));
  const int64_t tiles = (nvec + p.vt - 1) / p.vt;
  dim3 grid((unsigned)tmin<int64_t>(tiles, (int64_t)sms * occ), 2);
  fn<<<grid, kAppendThreads, smem, st>>>(p);
  return check_launch("tq_append");
}

int launch_dequant(const tq_geom* G, const tq_tables* t, const tq_cache* c,
                   int64_t t0, int64_t t1, const tq_tensor4* ko, const tq_tensor4* vo,
                   cudaStream_t st) {
  DequantParams p;
  p.g = make_geom(G->head_dim, G->key_bits, G->value_bits, G->qjl);
  p.cent[0] = t->k_centroids; p.cent[1] = t->v_centroids;
  p.R = t->rot;
  p.pages = c->pages; p.pm = page_map(c); p.status = device_status_word();
  const tq_tensor4* o[2] = {ko, vo};
  p.H = 1;
  for (int w = 0; w < 2; ++w) {
    p.out[w] = o[w] ? o[w]->data : nullptr;
    p.dtype[w] = o[w] ? o[w]->dtype : 0;
    for (int i = 0; i < 4; ++i) p.stride[w][i] = o[w] ? o[w]->stride[i] : 0;
    if (o[w]) p.H = o[w]->shape[1];
  }
  p.t0 = t0; p.t1 = t1;
  if (t1 <= t0) return TQ_OK;
  dim3 grid((unsigned)((t1 - t0 + kVT - 1) / kVT), (unsigned)c->streams, 2);
  size_t smem = (size_t)(kVT * p.g.D + kVT) * 4;
  dequant_kernel<<<grid, 128, smem, st>>>(p);
  return check_launch("tq_dequantize");
}

}  // namespace tq
