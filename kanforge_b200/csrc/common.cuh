// Shared host/device helpers of libkanb200: error reporting, the device error
// word written by bounded waits, and small math helpers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>
#include <cstdio>
#include <string>

#include "../../include/kanforge_b200.h"

namespace kf {

// ---- host-side error state (one message per calling thread) ---------------

void set_error(const char* fmt, ...);
void clear_error();

#define KF_CHECK_ARG(cond, ...)            \
  do {                                     \
    if (!(cond)) {                         \
      ::kf::set_error(__VA_ARGS__);        \
      return KF_ERR_ARG;                   \
    }                                      \
  } while (0)

#define KF_CUDA_RET(expr)                                                            \
  do {                                                                               \
    cudaError_t err__ = (expr);                                                      \
    if (err__ != cudaSuccess) {                                                      \
      ::kf::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(err__),     \
                      __FILE__, __LINE__);                                           \
      return KF_ERR_CUDA;                                                            \
    }                                                                                \
  } while (0)

// Checks the launch that was just enqueued.
int check_launch(const char* what);

// Makes the device that owns `ptr` current for this host thread in the
// library's (statically linked) CUDA runtime and binds its primary context.
// Every entry point calls it: callers such as torch's autograd engine launch
// from worker threads on which this runtime has never run, and a process may
// drive several GPUs.
int bind_device(const void* ptr);

// ---- device error word ----------------------------------------------------
// Bit set by a kernel whose bounded wait ran out; read and cleared by
// kf_device_status().  Kernels never trap: they record and return.
#define KF_DEVERR_MBAR_TIMEOUT 1
#define KF_DEVERR_BAD_SHAPE 2

// Without relocatable device code every translation unit owns its copy of the
// word; each registers a host reader so kf_device_status() can collect them all.
static __device__ int32_t g_device_error = 0;

__device__ __forceinline__ void report_device_error(int32_t bits) { atomicOr(&g_device_error, bits); }

using DeviceErrorReader = int (*)(int32_t*);
void register_device_error_reader(DeviceErrorReader fn);

// Reads and clears this translation unit's word.
static int read_device_error_word(int32_t* out) {
  int32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return KF_ERR_CUDA;
  const int32_t zero = 0;
  if (cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)) != cudaSuccess) return KF_ERR_CUDA;
  *out |= v;
  return KF_OK;
}

namespace {
struct DeviceErrorRegistration {
  DeviceErrorRegistration() { register_device_error_reader(&read_device_error_word); }
};
static DeviceErrorRegistration g_device_error_registration;
}  // namespace

// ---- small math ------------------------------------------------------------

__host__ __device__ __forceinline__ int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

}  // namespace kf
