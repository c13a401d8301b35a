// Host-side plumbing shared by the hive_b200 translation units: status codes and the
// per-thread "last error" message that every C-ABI entry point sets on failure.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>

#include "../../include/hive_b200.h"

namespace hv {

void set_error(const char* fmt, ...);
int cuda_fail(const char* what, cudaError_t e);
int sm_count(int* out);

// The reference-order decode attention (attn_exact.cuh, kernels in k_ops.cu), shared by
// hv_attn_decode, the batched prefill rows and the allocation-free entry point.
int ref_blas_runs();
int set_ref_blas_runs(int v);
int attn_exact_chunks(int nkv, int cap, int* out);
size_t attn_exact_scratch_floats(int nq, int cap, int nch);
int attn_exact_launch(int group, bool kv_half, const float* q, size_t q_tok, const void* kc,
                      const void* vc, float* ctx, size_t ctx_tok, const float* scale,
                      const int32_t* pos_p, int pos0, int nq, int cap, int nch, int ntok,
                      float* scr, size_t scr_tok, cudaStream_t st);

}  // namespace hv

#define HV_CUDA(call)                                         \
  do {                                                        \
    cudaError_t _e = (call);                                  \
    if (_e != cudaSuccess) return ::hv::cuda_fail(#call, _e); \
  } while (0)

#define HV_REQUIRE(cond, code, ...)          \
  do {                                       \
    if (!(cond)) {                           \
      ::hv::set_error(__VA_ARGS__);          \
      return (code);                         \
    }                                        \
  } while (0)

#define HV_LAUNCHED(name)                                         \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return ::hv::cuda_fail(name, _e);      \
    return HV_OK;                                                 \
  } while (0)
