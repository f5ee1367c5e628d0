// tq_internal.h — host-side glue shared by the .cu translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tq_b200.h"

namespace tq {

// Thread-local error message (tq_last_error).
void set_error(const char* fmt, ...);
// Returns TQ_OK, or TQ_ERR_CUDA with the launch error recorded.
int check_launch(const char* what);
// Same for the return code of an explicit launch (cudaLaunchKernelEx).
int launch_result(cudaError_t e, const char* what);
int set_smem_attr(const void* kernel, size_t bytes);
int device_sm_count();
// Resident CTAs per SM for a kernel (cached per device).
int occupancy(const void* kernel, int threads, size_t smem);

int launch_quantize_rotated(const float* y, int64_t n, const float* b, int nb,
                            int16_t* codes, cudaStream_t st);
int launch_append(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                  const tq_tensor4* k, const tq_tensor4* v, int64_t pos,
                  cudaStream_t st);
// Tensor-core append (head_dim 128, bf16 inputs, no QJL): TQ_OK when it ran,
// 1 when it does not apply (the caller uses the CUDA-core kernel), or an error.
int launch_append_tc(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                     const tq_tensor4* k, const tq_tensor4* v, int64_t pos, cudaStream_t st);
bool append_tc_applies(const tq_geom* g, const tq_tables* t, const tq_tensor4* k,
                       const tq_tensor4* v);
int read_tc_status(uint32_t* out, cudaStream_t st);
// Device address of the library status word read by tq_device_status.
uint32_t* device_status_word();
bool prefill_supported(int D, int kb, int vb);
// tcgen05 prefill attention (tq_prefill_tc.cu): TQ_OK when it ran, 1 when it
// does not apply (the caller uses the mma.sync kernel), or an error.
int launch_prefill_tc(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                      const tq_prefill_args* a, uint32_t* status, cudaStream_t st);
bool prefill_tc_applies(const tq_geom* g);
int launch_prefill(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                   const tq_prefill_args* a, uint32_t* status, cudaStream_t st);
int launch_dequant(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                   int64_t t0, int64_t t1, const tq_tensor4* ko, const tq_tensor4* vo,
                   cudaStream_t st);
size_t decode_workspace_bytes(const tq_geom* g, const tq_cache* c,
                              const tq_decode_args* a);
// The new token of a decode step (tq_decode_step): stored at `pos` by the
// query-preparation kernel before attention.
struct StepInput {
  const tq_tensor4* k;
  const tq_tensor4* v;
  int64_t pos;
};
int launch_decode(const tq_geom* g, const tq_tables* t, const tq_cache* c,
                  const tq_decode_args* a, void* ws, size_t ws_bytes, cudaStream_t st,
                  const StepInput* step = nullptr);

// cudaLaunchKernelEx with programmatic stream serialisation (see pdl_wait).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

}  // namespace tq
