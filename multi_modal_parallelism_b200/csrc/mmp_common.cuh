// Shared helpers for the sm_100a kernels of libmmp_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "mmp_b200.h"

namespace mmp {

using bf16 = __nv_bfloat16;

// Device error bits (OR-ed into the caller's error word; the kernels never trap).
enum : int {
  DEVERR_INDEX = 1,      // a state line / slot / block index outside its buffer
  DEVERR_POSITION = 2,   // a RoPE position outside the cos/sin table
  DEVERR_TIMEOUT = 4,    // a bounded wait ran out
};

__device__ __forceinline__ void flag_error(int* err, int bits) {
  if (err) atomicOr(err, bits);
}

__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }

// Two bf16 packed in a 32-bit word <-> float2.
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 16-byte global accesses with streaming (evict-first) cache hints.
__device__ __forceinline__ uint4 ld_stream16(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ void st_stream16(void* p, uint4 v) { __stcs(reinterpret_cast<uint4*>(p), v); }
// L2 prefetch of `bytes` contiguous bytes (16-byte aligned address, bytes a multiple of 16); a hint: no data is
// returned and nothing completes.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint4 ld16(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void st16(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

// x * sigmoid(x) with the fast divide (2 ulp; x / inf -> 0 for very negative x): outputs are bf16
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.f + __expf(-x)); }

__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(__expf(x)); }

template <int WIDTH = 32>
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` is >= 32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

__host__ __device__ inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch. Every kernel lets the next kernel in the stream start launching as soon as
// all of its own CTAs are running (pdl_trigger), and waits for the previous kernel to finish and flush its
// memory (pdl_wait) before touching anything that kernel may have written.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// bit 0: tensor-core GEMMs, bit 1: every other kernel
bool pdl_enabled(int kind = 2);

// Launch with the programmatic-stream-serialization attribute (when enabled) plus optional extra attributes.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kind(int kind, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                               const cudaLaunchAttribute* extra, int n_extra, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[4];
  int n = 0;
  for (int i = 0; i < n_extra && n < 3; ++i) attr[n++] = extra[i];
  if (pdl_enabled(kind)) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                          const cudaLaunchAttribute* extra, int n_extra, Args&&... args) {
  return launch_kind(2, kern, grid, block, smem, s, extra, n_extra, std::forward<Args>(args)...);
}

}  // namespace mmp

// Host-side status helpers shared by every entry point.
int mmp_set_error(int code, const char* fmt, ...);
int mmp_check_launch(const char* what);
