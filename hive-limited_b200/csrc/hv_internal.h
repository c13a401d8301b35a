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
