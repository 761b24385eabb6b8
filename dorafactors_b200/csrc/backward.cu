// Fused DoRA compose backward for sm_100a: one pass over d_out (and inner).
//
//   d_lora = (g * s) * d_out
//   d_base = (g - 1) * d_out
//   d_g    = sum over rows of inner * d_out        (per column)
//
// Same thread layout as the forward: a thread owns one 16-byte column slice
// and walks down a strided set of rows, so g and the running d_g sums of its
// columns live in registers.  The column sum is reduced deterministically:
//   1. each thread accumulates its rows serially in fp32;
//   2. the CTA folds its row-threads through shared memory in a fixed order;
//   3. every CTA writes its column partial to the workspace, and the last CTA
//      to finish a column tile (a completion counter, no spin-waits) folds the
//      partials of all CTAs in blockIdx.y order and writes d_g.
// No float atomics are used, so repeated calls give identical bits.
#include "dora_common.cuh"

namespace dora {

// kRG selects the layer-output form: the second gradient is d_result = g * d_y
// (the base branch of y = result + delta) instead of d_base = (g - 1) * d_out.
// At most 80 registers (three 256-thread CTAs per SM): more loads in flight per SM.
// kLd: d_out rows are ld_d elements apart (a column slice of a wider gradient,
// the row-sharded layer's share of the full d_y); every other array is dense.
template <typename TA, typename TG, int VEC, bool kDL, bool kDB, bool kDG, bool kRG, bool kLd>
__global__ void __launch_bounds__(256, 3)
compose_bwd_kernel(const TA* __restrict__ d_out, const TA* __restrict__ inner, const TG* __restrict__ g, float s,
                   TA* __restrict__ d_lora, TA* __restrict__ d_base, TG* __restrict__ d_g,
                   unsigned* __restrict__ counters, float* __restrict__ partials, int64_t rows, int64_t vcols,
                   int64_t ld_d) {
  __shared__ float red[256 * VEC];
  __shared__ bool is_last;
  const int64_t vc = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool active = vc < vcols;
  const int64_t cols = vcols * VEC;
  float gs[VEC], gm1[VEC], acc[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    const float gv = active ? to_f32(g[vc * VEC + k]) : 0.f;
    gs[k] = __fmul_rn(gv, s);
    gm1[k] = kRG ? gv : __fsub_rn(gv, 1.0f);
    acc[k] = 0.f;
  }
  const int64_t row0 = int64_t(blockIdx.y) * blockDim.y + threadIdx.y;
  const int64_t rstep = int64_t(gridDim.y) * blockDim.y;
  constexpr int U = 4;
  if (active) {
    for (int64_t r = row0; r < rows; r += U * rstep) {
      if constexpr (VEC > 1) {
        uint4 dv[U], iv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t rr = r + u * rstep;
          if (rr < rows) {
            const int64_t off = rr * cols + vc * VEC;
            dv[u] = ld_stream(d_out + (kLd ? rr * ld_d + vc * VEC : off));
            if constexpr (kDG) iv[u] = ld_stream(inner + off);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t rr = r + u * rstep;
          if (rr < rows) {
            const int64_t off = rr * cols + vc * VEC;
            float df[VEC], xf[VEC], lf[VEC], bf[VEC];
            Vec16<TA>::unpack(dv[u], df);
            if constexpr (kDG) Vec16<TA>::unpack(iv[u], xf);
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
              if constexpr (kDL) lf[k] = __fmul_rn(gs[k], df[k]);
              if constexpr (kDB) bf[k] = __fmul_rn(gm1[k], df[k]);
              if constexpr (kDG) acc[k] = fmaf(xf[k], df[k], acc[k]);
            }
            // Streaming stores (evict-first): same GPU, 16384 x 28672 0.6075 -> 0.6031 ms,
            // 8192 x 8192 0.1015 -> 0.0985 ms.
            if constexpr (kDL) st_stream(d_lora + off, Vec16<TA>::pack(lf));
            if constexpr (kDB) st_stream(d_base + off, Vec16<TA>::pack(bf));
          }
        }
      } else {
        float df[U], xf[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t rr = r + u * rstep;
          if (rr < rows) {
            df[u] = to_f32(d_out[(kLd ? rr * ld_d : rr * cols) + vc]);
            if constexpr (kDG) xf[u] = to_f32(inner[rr * cols + vc]);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t rr = r + u * rstep;
          if (rr < rows) {
            if constexpr (kDL) d_lora[rr * cols + vc] = from_f32<TA>(__fmul_rn(gs[0], df[u]));
            if constexpr (kDB) d_base[rr * cols + vc] = from_f32<TA>(__fmul_rn(gm1[0], df[u]));
            if constexpr (kDG) acc[0] = fmaf(xf[u], df[u], acc[0]);
          }
        }
      }
    }
  }
  if constexpr (kDG) {
    const int tx = threadIdx.x, ty = threadIdx.y, TX = blockDim.x, TY = blockDim.y;
#pragma unroll
    for (int k = 0; k < VEC; ++k) red[(ty * TX + tx) * VEC + k] = acc[k];
    __syncthreads();
    if (ty == 0 && active) {
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        float t = red[tx * VEC + k];
        for (int y = 1; y < TY; ++y) t += red[(y * TX + tx) * VEC + k];
        partials[int64_t(blockIdx.y) * cols + vc * VEC + k] = t;
      }
    }
    __threadfence();
    __syncthreads();
    if (tx == 0 && ty == 0) {
      const unsigned done = atomicAdd(&counters[blockIdx.x], 1u);
      is_last = (done == gridDim.y - 1);
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      // All threads of the last CTA fold the tile's columns, consecutive threads on
      // consecutive columns (coalesced partial reads), loads issued eight row-blocks
      // at a time; the additions keep blockIdx.y order.
      const int lin = ty * TX + tx, nthr = TX * TY;
      const int64_t c0 = int64_t(blockIdx.x) * TX * VEC;
      for (int j = lin; j < TX * VEC; j += nthr) {
        const int64_t c = c0 + j;
        if (c >= cols) break;
        float t = 0.f;
        unsigned y = 0;
        for (; y + 8 <= gridDim.y; y += 8) {
          float v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) v[q] = __ldcg(partials + int64_t(y + q) * cols + c);
#pragma unroll
          for (int q = 0; q < 8; ++q) t += v[q];
        }
        for (; y < gridDim.y; ++y) t += __ldcg(partials + int64_t(y) * cols + c);
        d_g[c] = from_f32<TG>(t);
      }
      if (tx == 0 && ty == 0) counters[blockIdx.x] = 0u;  // ready for the next call
    }
  }
}

struct BwdPlan {
  bool vec;
  int64_t vcols;
  EwShape sh;
  size_t counter_bytes, partial_bytes;
};

// Row-grid depth: about 40 rows per thread, between the depths of 8 and of 32 CTAs
// per SM's worth.  Deeper grids balance the SMs better; every grid row adds a row of
// column partials that the last CTA of each column tile folds at the end.  Same GPU,
// layer-output form: 16384 x 28672 0.631 (8 per SM) / 0.617 (16) / 0.610 ms (32);
// 8192 x 8192 0.1015 / 0.108 / 0.125 ms.  shallow = true keeps the 8-per-SM depth
// (fewer partials, for a fixed-size scratch).
static BwdPlan bwd_plan(int64_t rows, int64_t cols, int esize, bool aligned, bool shallow = false) {
  BwdPlan p;
  const int V = 16 / esize;
  p.vec = aligned && (cols % V == 0);
  p.vcols = p.vec ? cols / V : cols;
  p.sh = ew_shape(rows, p.vcols, 8);
  if (!shallow) {
    const int64_t deep = ew_shape(rows, p.vcols, 32).grid.y;
    int64_t gy = rows / 160;
    if (gy > deep) gy = deep;
    if (gy > int64_t(p.sh.grid.y)) p.sh.grid.y = unsigned(gy);
  }
  p.counter_bytes = ((size_t(p.sh.grid.x) * 4 + 255) / 256) * 256;
  p.partial_bytes = size_t(p.sh.grid.y) * size_t(cols) * 4;
  return p;
}

template <typename TA, typename TG, int V, bool DL, bool DB, bool DG, bool RG, bool LD>
static void launch_bwd_v(const BwdPlan& p, const void* d_out, const void* inner, const void* g, float s,
                         void* d_lora, void* d_base, void* d_g, unsigned* cnt, float* part, int64_t rows,
                         int64_t ld_d, cudaStream_t st) {
  compose_bwd_kernel<TA, TG, V, DL, DB, DG, RG, LD><<<p.sh.grid, p.sh.block, 0, st>>>(
      static_cast<const TA*>(d_out), static_cast<const TA*>(inner), static_cast<const TG*>(g), s,
      static_cast<TA*>(d_lora), static_cast<TA*>(d_base), static_cast<TG*>(d_g), cnt, part, rows, p.vcols, ld_d);
}

template <typename TA, typename TG, int V, bool RG, bool LD>
static void launch_bwd_sel(const BwdPlan& p, const void* d_out, const void* inner, const void* g, float s,
                           void* d_lora, void* d_base, void* d_g, unsigned* cnt, float* part, int64_t rows,
                           int64_t ld_d, cudaStream_t st) {
  const int sel = (d_lora ? 4 : 0) | (d_base ? 2 : 0) | (d_g ? 1 : 0);
#define DORA_BWD_CASE(n, a, b, c) \
  case n: launch_bwd_v<TA, TG, V, a, b, c, RG, LD>(p, d_out, inner, g, s, d_lora, d_base, d_g, cnt, part, rows, \
                                                   ld_d, st); break;
  switch (sel) {
    DORA_BWD_CASE(1, false, false, true)
    DORA_BWD_CASE(2, false, true, false)
    DORA_BWD_CASE(3, false, true, true)
    DORA_BWD_CASE(4, true, false, false)
    DORA_BWD_CASE(5, true, false, true)
    DORA_BWD_CASE(6, true, true, false)
    DORA_BWD_CASE(7, true, true, true)
    default: break;
  }
#undef DORA_BWD_CASE
}

template <typename TA, typename TG, bool RG, bool LD = false>
static int launch_bwd(const void* d_out, const void* inner, const void* g, float s, void* d_lora, void* d_base,
                      void* d_g, void* ws, size_t ws_bytes, int64_t rows, int64_t cols, cudaStream_t st,
                      int64_t ld_d = 0, bool shallow = false) {
  constexpr int V = 16 / sizeof(TA);
  const bool aligned = aligned16(d_out) && (!inner || aligned16(inner)) && (!d_lora || aligned16(d_lora)) &&
                       (!d_base || aligned16(d_base)) && (!LD || ld_d % V == 0);
  BwdPlan p = bwd_plan(rows, cols, sizeof(TA), aligned, shallow);
  unsigned* cnt = nullptr;
  float* part = nullptr;
  if (d_g) {
    if (!ws || ws_bytes < p.counter_bytes + p.partial_bytes || (reinterpret_cast<uintptr_t>(ws) & 255u))
      return DORA_ERR_WORKSPACE;
    cnt = static_cast<unsigned*>(ws);
    part = reinterpret_cast<float*>(static_cast<char*>(ws) + p.counter_bytes);
  }
  if (p.vec) launch_bwd_sel<TA, TG, V, RG, LD>(p, d_out, inner, g, s, d_lora, d_base, d_g, cnt, part, rows, ld_d, st);
  else launch_bwd_sel<TA, TG, 1, RG, LD>(p, d_out, inner, g, s, d_lora, d_base, d_g, cnt, part, rows, ld_d, st);
  return check_launch();
}

}  // namespace dora

using namespace dora;

extern "C" size_t dora_compose_bwd_workspace_size(int64_t rows, int64_t cols, int act_dtype) {
  if (rows <= 0 || cols <= 0 || !dtype_ok(act_dtype)) return 0;
  // The unaligned plan has the most column tiles, so it bounds both layouts.
  BwdPlan a = bwd_plan(rows, cols, dtype_size(act_dtype), true);
  BwdPlan b = bwd_plan(rows, cols, dtype_size(act_dtype), false);
  size_t na = a.counter_bytes + a.partial_bytes, nb = b.counter_bytes + b.partial_bytes;
  return na > nb ? na : nb;
}

namespace dora {

template <bool RG, bool LD = false>
static int bwd_entry(const void* d_out, const void* inner, const void* g, int g_dtype, double scale, void* d_lora,
                     void* d_base, void* d_g, void* workspace, size_t workspace_bytes, int64_t rows, int64_t cols,
                     int act_dtype, void* stream, int64_t ld_d = 0, bool shallow = false) {
  if (rows < 0 || cols < 0 || !dtype_ok(act_dtype) || !dtype_ok(g_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (LD && ld_d < cols) return DORA_ERR_INVALID_ARGUMENT;
  if (!d_lora && !d_base && !d_g) return DORA_OK;
  if (rows == 0 || cols == 0) {
    // Empty activations (their pointers may be null, as PyTorch gives for zero
    // elements): the column sums are zero, the reference's result for an empty
    // batch (test_dora_fused.py TestEdgeCases, empty-tensor backward).
    if (d_g && cols > 0) {
      cudaError_t e = cudaMemsetAsync(d_g, 0, size_t(cols) * dtype_size(g_dtype), static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return set_cuda_error(e);
    }
    return DORA_OK;
  }
  if (d_g && !inner) return DORA_ERR_INVALID_ARGUMENT;
  if (!d_out || !g) return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float s = float(scale);
  switch (act_dtype) {
    case DORA_DTYPE_BF16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_bwd<__nv_bfloat16, float, RG, LD>(d_out, inner, g, s, d_lora, d_base, d_g, workspace,
                                                            workspace_bytes, rows, cols, st, ld_d, shallow)
                 : launch_bwd<__nv_bfloat16, __nv_bfloat16, RG, LD>(d_out, inner, g, s, d_lora, d_base, d_g,
                                                                    workspace, workspace_bytes, rows, cols, st, ld_d, shallow);
    case DORA_DTYPE_F16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_bwd<__half, float, RG, LD>(d_out, inner, g, s, d_lora, d_base, d_g, workspace,
                                                     workspace_bytes, rows, cols, st, ld_d, shallow)
                 : launch_bwd<__half, __half, RG, LD>(d_out, inner, g, s, d_lora, d_base, d_g, workspace,
                                                      workspace_bytes, rows, cols, st, ld_d, shallow);
    default:
      return launch_bwd<float, float, RG, LD>(d_out, inner, g, s, d_lora, d_base, d_g, workspace, workspace_bytes,
                                              rows, cols, st, ld_d, shallow);
  }
}

}  // namespace dora

extern "C" int dora_compose_bwd(const void* d_out, const void* inner, const void* g, int g_dtype, double scale,
                                void* d_lora, void* d_base, void* d_g, void* workspace, size_t workspace_bytes,
                                int64_t rows, int64_t cols, int act_dtype, void* stream) {
  return bwd_entry<false>(d_out, inner, g, g_dtype, scale, d_lora, d_base, d_g, workspace, workspace_bytes, rows,
                          cols, act_dtype, stream);
}

extern "C" int dora_linear_output_bwd(const void* d_y, const void* inner, const void* g, int g_dtype, double scale,
                                      void* d_lora, void* d_result, void* d_g, void* workspace,
                                      size_t workspace_bytes, int64_t rows, int64_t cols, int act_dtype,
                                      void* stream) {
  return bwd_entry<true>(d_y, inner, g, g_dtype, scale, d_lora, d_result, d_g, workspace, workspace_bytes, rows,
                         cols, act_dtype, stream);
}

extern "C" int dora_linear_output_bwd_strided(const void* d_y, int64_t ld_dy, const void* inner, const void* g,
                                              int g_dtype, double scale, void* d_lora, void* d_result, void* d_g,
                                              void* workspace, size_t workspace_bytes, int64_t rows, int64_t cols,
                                              int act_dtype, void* stream) {
  return bwd_entry<true, true>(d_y, inner, g, g_dtype, scale, d_lora, d_result, d_g, workspace, workspace_bytes,
                               rows, cols, act_dtype, stream, ld_dy);
}

// ---------------------------------------------------------------------------
// Bias gradient of the layer-output form: y depends on the bias only through
// base = result - bias, so d_bias[j] = -sum_i (g[j] - 1) * d_y[i, j]
// = (1 - g[j]) * sum_i d_y[i, j].  One CTA per 64 columns (eight 16-byte
// column vectors x 32 row lanes for 16-bit types), rows summed serially per
// thread in fp32 and folded across the 32 lanes in a fixed order: deterministic,
// no workspace, one read of d_y.
// ---------------------------------------------------------------------------
namespace dora {

template <typename TA, typename TG, int VEC>
__global__ void __launch_bounds__(256) bias_grad_kernel(const TA* __restrict__ d_y, const TG* __restrict__ g,
                                                        TA* __restrict__ d_bias, int64_t rows, int64_t vcols) {
  __shared__ float red[32][8 * VEC + 1];
  const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;  // 8 column vectors x 32 row lanes
  const int64_t vc = int64_t(blockIdx.x) * 8 + tx;
  const int64_t cols = vcols * VEC;
  float acc[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) acc[k] = 0.f;
  if (vc < vcols) {
    for (int64_t r = ty; r < rows; r += 32) {
      if constexpr (VEC > 1) {
        float f[VEC];
        Vec16<TA>::unpack(ld_stream(d_y + r * cols + vc * VEC), f);
#pragma unroll
        for (int k = 0; k < VEC; ++k) acc[k] += f[k];
      } else {
        acc[0] += to_f32(d_y[r * cols + vc]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < VEC; ++k) red[ty][tx * VEC + k] = acc[k];
  __syncthreads();
  if (threadIdx.x < 8 * VEC) {
    const int j = threadIdx.x;
    const int64_t c = int64_t(blockIdx.x) * 8 * VEC + j;
    if (c < cols) {
      float t = 0.f;
      for (int y = 0; y < 32; ++y) t += red[y][j];
      d_bias[c] = from_f32<TA>(__fmul_rn(__fsub_rn(1.0f, to_f32(g[c])), t));
    }
  }
}

template <typename TA, typename TG>
static int launch_bias_grad(const void* d_y, const void* g, void* d_bias, int64_t rows, int64_t cols,
                            cudaStream_t st) {
  constexpr int V = 16 / sizeof(TA);
  const bool vec = cols % V == 0 && aligned16(d_y);
  const int64_t vcols = vec ? cols / V : cols;
  const int64_t grid = (vcols + 7) / 8;
  if (grid > int64_t(INT32_MAX)) return DORA_ERR_UNSUPPORTED;
  if (vec)
    bias_grad_kernel<TA, TG, V><<<unsigned(grid), 256, 0, st>>>(static_cast<const TA*>(d_y),
                                                                 static_cast<const TG*>(g), static_cast<TA*>(d_bias),
                                                                 rows, vcols);
  else
    bias_grad_kernel<TA, TG, 1><<<unsigned(grid), 256, 0, st>>>(static_cast<const TA*>(d_y),
                                                                 static_cast<const TG*>(g), static_cast<TA*>(d_bias),
                                                                 rows, vcols);
  return check_launch();
}

}  // namespace dora

extern "C" int dora_linear_output_bias_grad(const void* d_y, const void* g, int g_dtype, void* d_bias, int64_t rows,
                                            int64_t cols, int act_dtype, void* stream) {
  if (rows < 0 || cols < 0 || !dtype_ok(act_dtype) || !dtype_ok(g_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (cols == 0) return DORA_OK;
  if (!d_bias || !g || (rows > 0 && !d_y)) return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    cudaError_t e = cudaMemsetAsync(d_bias, 0, size_t(cols) * dtype_size(act_dtype), st);
    return e == cudaSuccess ? DORA_OK : set_cuda_error(e);
  }
  switch (act_dtype) {
    case DORA_DTYPE_BF16:
      return g_dtype == DORA_DTYPE_F32 ? launch_bias_grad<__nv_bfloat16, float>(d_y, g, d_bias, rows, cols, st)
                                       : launch_bias_grad<__nv_bfloat16, __nv_bfloat16>(d_y, g, d_bias, rows, cols, st);
    case DORA_DTYPE_F16:
      return g_dtype == DORA_DTYPE_F32 ? launch_bias_grad<__half, float>(d_y, g, d_bias, rows, cols, st)
                                       : launch_bias_grad<__half, __half>(d_y, g, d_bias, rows, cols, st);
    default:
      return launch_bias_grad<float, float>(d_y, g, d_bias, rows, cols, st);
  }
}

// ---------------------------------------------------------------------------
// Allocation-free variant of dora_compose_bwd.
//
// Some callers cannot hand this library a device workspace: a C or FFI host
// that embeds the library without any device allocator of its own, or code
// that must not call cudaMalloc on this path because cudaMalloc synchronizes
// the device.  For them the column-sum scratch lives in a fixed array in this
// library's device image instead.  The array exists once per GPU that loads
// the library and stays allocated until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace dora {

constexpr size_t kStaticScratchBytes = size_t(DORA_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) unsigned char g_bwd_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
static std::mutex g_scratch_mutex;
static void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_bwd_scratch on the current device.  In host code the
// symbol's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.  The cache is never
// invalidated: after cudaDeviceReset the cached address belongs to the old
// context, so this entry point must not be used across a device reset.
static int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  if (dev < 0 || dev >= kMaxDevices) return DORA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess) return set_cuda_error(e);
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return DORA_OK;
}

}  // namespace dora

extern "C" int dora_compose_bwd_noalloc(const void* d_out, const void* inner, const void* g, int g_dtype,
                                        double scale, void* d_lora, void* d_base, void* d_g, int64_t rows,
                                        int64_t cols, int act_dtype, void* stream) {
  if (rows < 0 || cols < 0 || !dtype_ok(act_dtype) || !dtype_ok(g_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (!d_g || rows == 0 || cols == 0) {
    // No column sum (or nothing to sum over): no scratch is touched.
    return dora_compose_bwd(d_out, inner, g, g_dtype, scale, d_lora, d_base, d_g, nullptr, 0, rows, cols,
                            act_dtype, stream);
  }
  // The workspace entry point's grid when its column partials fit the fixed array,
  // else the shallow one (8 CTAs per SM's worth); beyond that the shape is rejected.
  auto need_at = [&](bool shallow) {
    const BwdPlan a = bwd_plan(rows, cols, dtype_size(act_dtype), true, shallow);
    const BwdPlan b = bwd_plan(rows, cols, dtype_size(act_dtype), false, shallow);
    const size_t na = a.counter_bytes + a.partial_bytes, nb = b.counter_bytes + b.partial_bytes;
    return na > nb ? na : nb;
  };
  bool shallow = false;
  if (need_at(false) > kStaticScratchBytes) shallow = true;
  if (need_at(true) > kStaticScratchBytes) return DORA_ERR_WORKSPACE;
  // The rest of dora_compose_bwd's argument checks run before the array is
  // touched, so a call that will be rejected queues nothing on it.
  if (!inner || !d_out || !g) return DORA_ERR_INVALID_ARGUMENT;
  void* ws = nullptr;
  int rc = static_scratch_address(&ws);
  if (rc != DORA_OK) return rc;
  // The scratch keeps whatever the last call left in it.  Only the completion
  // counters at its start must begin at zero; clear them on this stream (the
  // column partials are always written before they are read).
  const size_t c_vec = bwd_plan(rows, cols, dtype_size(act_dtype), true).counter_bytes;
  const size_t c_any = bwd_plan(rows, cols, dtype_size(act_dtype), false).counter_bytes;
  const size_t counter_bytes = c_vec > c_any ? c_vec : c_any;
  cudaError_t e = cudaMemsetAsync(ws, 0, counter_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_cuda_error(e);
  return bwd_entry<false>(d_out, inner, g, g_dtype, scale, d_lora, d_base, d_g, ws, kStaticScratchBytes, rows, cols,
                          act_dtype, stream, 0, shallow);
}
