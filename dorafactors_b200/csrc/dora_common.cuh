// Shared device/host helpers for the DoRA sm_100a kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dora_b200.h"

namespace dora {

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<DORA_DTYPE_F32> {
  using T = float;
  static constexpr int kVec = 4;  // elements per 16-byte vector
};
template <> struct Elem<DORA_DTYPE_F16> {
  using T = __half;
  static constexpr int kVec = 8;
};
template <> struct Elem<DORA_DTYPE_BF16> {
  using T = __nv_bfloat16;
  static constexpr int kVec = 8;
};

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

inline int dtype_size(int dt) {
  switch (dt) {
    case DORA_DTYPE_F32: return 4;
    case DORA_DTYPE_F16: return 2;
    case DORA_DTYPE_BF16: return 2;
    default: return 0;
  }
}
inline bool dtype_ok(int dt) { return dtype_size(dt) != 0; }

// 16-byte vector of elements unpacked to / packed from fp32.
template <typename T> struct Vec16;
template <> struct Vec16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};
template <typename H> struct Vec16Half {
  static constexpr int N = 8;
  __device__ __forceinline__ static void unpack(const uint4& v, float (&f)[8]) {
    const H* h = reinterpret_cast<const H*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
  }
  __device__ __forceinline__ static uint4 pack(const float (&f)[8]) {
    uint4 v;
    H* h = reinterpret_cast<H*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<H>(f[i]);
    return v;
  }
};
template <> struct Vec16<__half> : Vec16Half<__half> {};
template <> struct Vec16<__nv_bfloat16> : Vec16Half<__nv_bfloat16> {};

// Streaming 16-byte global accesses.  Inputs of the elementwise kernels are
// read exactly once, so they bypass L1.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_stream_coherent(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_global(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
// Streaming store (evict-first in L2): outputs that the kernel never reads again and
// that are far larger than L2.
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------
// Device error word: set by a kernel whose bounded wait expired.
// ---------------------------------------------------------------------------
extern __device__ int g_device_error;
__device__ __forceinline__ void record_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ---------------------------------------------------------------------------
// Host helpers
// ---------------------------------------------------------------------------
int set_cuda_error(cudaError_t e);  // records the text, returns DORA_ERR_CUDA
void count_launches(int n);         // adds to the library-wide launch counter
// Call after every kernel launch: counts it and reports launch errors.
inline int check_launch(int launches = 1) {
  count_launches(launches);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DORA_OK : set_cuda_error(e);
}

// Programmatic dependent launch.  A kernel started with launch_pdl may begin while
// the previous kernel in the stream is still running (its prologue overlaps that
// kernel's tail); it calls pdl_wait() before touching anything the previous
// kernel writes.  pdl_trigger() lets the next such kernel start early.  Both are
// no-ops in a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// SM count of the current device, looked up once per device.
inline int num_sms() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = cache[dev];  // every writer stores the same value
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return n;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch shape shared by the elementwise kernels: blockDim = (tx, 256 / tx),
// tx threads across 16-byte column slices, the rest across rows; about eight
// 256-thread CTAs per SM in total.
struct EwShape {
  dim3 grid, block;
};
inline EwShape ew_shape(int64_t rows, int64_t vcols, int ctas_per_sm = 8) {
  int tx = 32;
  while (tx < 64 && tx < vcols) tx *= 2;
  const int ty = 256 / tx;
  const int64_t gx = (vcols + tx - 1) / tx;
  const int64_t target = int64_t(num_sms()) * ctas_per_sm;
  int64_t gy = (target + gx - 1) / gx;
  const int64_t need = (rows + ty - 1) / ty;
  if (gy > need) gy = need;
  if (gy < 1) gy = 1;
  if (gy > 65535) gy = 65535;
  EwShape sh;
  sh.grid = dim3(unsigned(gx), unsigned(gy), 1);
  sh.block = dim3(unsigned(tx), unsigned(ty), 1);
  return sh;
}

// Grid of the streaming elementwise kernels whose threads walk down the rows in
// groups of four: deep (up to 64 CTAs per SM's worth, so CTAs retire and refill evenly)
// but with at least three row groups per thread, and never shallower than 8 per SM.
inline EwShape ew_shape_deep(int64_t rows, int64_t vcols) {
  EwShape sh = ew_shape(rows, vcols, 8);
  const EwShape deep = ew_shape(rows, vcols, 64);
  const int64_t cap = rows / (int64_t(sh.block.y) * 4 * 3);
  const int64_t gy = int64_t(deep.grid.y) < cap ? int64_t(deep.grid.y) : cap;
  if (gy > int64_t(sh.grid.y)) sh.grid.y = unsigned(gy);
  return sh;
}

}  // namespace dora
