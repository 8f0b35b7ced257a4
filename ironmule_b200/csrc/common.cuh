// Shared helpers for the libimspec kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/imspec.h"

namespace im {

// ---- error reporting across the C ABI ---------------------------------------------------------
// Every entry point returns IM_OK (0) or a non-zero status (IM_UNSUPPORTED, IM_INVALID,
// IM_CUDA_ERROR) and leaves a message that im_last_error() returns on the calling thread.
void set_error(const char* fmt, ...);
void clear_error();

#define IM_REQUIRE(cond, code, ...)      \
  do {                                   \
    if (!(cond)) {                       \
      ::im::set_error(__VA_ARGS__);      \
      return (code);                     \
    }                                    \
  } while (0)

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return IM_CUDA_ERROR;
  }
  return IM_OK;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- programmatic dependent launch --------------------------------------------------------------
// Decode-path kernels are launched with programmatic stream serialisation: a kernel's CTAs may become
// resident while the previous kernel on the stream is still running. Every such kernel calls pdl_wait()
// before it reads anything an earlier kernel wrote and before its first global write (what comes before
// may only read weights, which no kernel on the decode path writes), and pdl_trigger() after it, which
// lets the next kernel's CTAs launch. pdl_wait() returns once the previous grid has completed and its
// writes are visible; for a kernel launched without the attribute it returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Process-wide switch (im_set_launch_overlap); on by default.
inline bool& launch_overlap() {
  static bool on = true;
  return on;
}

template <typename... KArgs, typename... Args>
inline int launch(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                  Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = launch_overlap() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return IM_CUDA_ERROR;
  }
  return IM_OK;
}

// ---- bf16 as raw 16-bit patterns --------------------------------------------------------------
// Values cross the ABI as uint16_t bit patterns; arithmetic is float32 with one rounding to bf16
// (nearest even) wherever the reference rounds.
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
__device__ __forceinline__ uint16_t to_bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
__device__ __forceinline__ float round_bf(float f) { return bf(to_bf(f)); }

// Streaming 8-byte load that does not allocate in L1 (weights are read once per launch).
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Cached read-only loads (activations that every CTA re-reads stay in L1).
__device__ __forceinline__ uint4 ldg_u4(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p) { return __ldg(p); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace im
