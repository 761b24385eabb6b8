// Fused DoRA compose forward for sm_100a.
//
// Delta form (the DoRA layer's return value, dora.py:1380-1484):
//   out   = (g - 1) * base + g * (s * lora)
//   inner = s * lora + base                      (training forward only)
// Layer-output form (the delta added to the base output in the same pass, the
// glue of DoraLinearVariant.forward, variants.py:244-283):
//   base  = result - bias                        (bias optional, per column)
//   y     = result + ((g - 1) * base + g * (s * lora))
//   inner = s * lora + base
//
// The kernel is HBM-bound (2 reads + 1 or 2 writes per element).  Each thread
// owns one 16-byte column slice of the [rows x cols] activation and walks down
// the rows, so the slices of g (and bias) it needs are loaded once into
// registers and reused for every row (no per-element g traffic, no index
// division).  A warp covers 32 consecutive 16-byte slices of one row (512
// contiguous bytes), and four rows are in flight per thread.  The grid is deep
// (64 CTAs per SM's worth, so each thread covers only a few row groups and CTAs
// retire and refill evenly) and the outputs use streaming stores.
//
// Arithmetic is fp32 with one rounding per output; the op order is the
// reference's ((g - 1) * base + g * (s * lora), dora_fused.py:32-54, then
// result + delta), each op correctly rounded (no FMA contraction), so fp32
// results are bitwise equal to the reference's fp32 PyTorch evaluation.
#include "dora_common.cuh"

namespace dora {

// kNc selects the read-only (non-coherent) load path; the in-place form
// (out == lora) reads with coherent loads instead, since lora is written.
// kOutput selects the layer-output form, kBias its bias subtraction.
template <typename TA, typename TG, int VEC, bool kInner, bool kNc, bool kOutput, bool kBias>
__global__ void __launch_bounds__(256)
compose_fwd_kernel(const TA* lora, const TA* __restrict__ base, const TG* __restrict__ g,
                   const TA* __restrict__ bias, float s, TA* out, TA* __restrict__ inner, int64_t rows,
                   int64_t vcols) {
  const int64_t vc = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;  // vector column
  if (vc >= vcols) return;
  const int64_t cols = vcols * VEC;
  float gv[VEC], gm1[VEC], bv[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) {
    gv[k] = to_f32(g[vc * VEC + k]);
    gm1[k] = __fsub_rn(gv[k], 1.0f);
    bv[k] = kBias ? to_f32(bias[vc * VEC + k]) : 0.f;
  }
  // One element: r is the second input (base, or the layer's result).
  auto one = [&](float l, float r, int k, float& o, float& in) {
    const float b = kBias ? __fsub_rn(r, bv[k]) : r;
    const float sl = __fmul_rn(s, l);
    const float d = __fadd_rn(__fmul_rn(gm1[k], b), __fmul_rn(gv[k], sl));
    o = kOutput ? __fadd_rn(r, d) : d;
    if constexpr (kInner) in = __fadd_rn(sl, b);
  };
  const int64_t row0 = int64_t(blockIdx.y) * blockDim.y + threadIdx.y;
  const int64_t rstep = int64_t(gridDim.y) * blockDim.y;
  constexpr int U = 4;  // rows in flight per thread
  for (int64_t r = row0; r < rows; r += U * rstep) {
    if constexpr (VEC > 1) {
      uint4 lv[U], rv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t rr = r + u * rstep;
        if (rr < rows) {
          const int64_t off = rr * cols + vc * VEC;
          lv[u] = kNc ? ld_stream(lora + off) : ld_stream_coherent(lora + off);
          rv[u] = ld_stream(base + off);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t rr = r + u * rstep;
        if (rr < rows) {
          const int64_t off = rr * cols + vc * VEC;
          float lf[VEC], bf[VEC], of[VEC], inf[VEC];
          Vec16<TA>::unpack(lv[u], lf);
          Vec16<TA>::unpack(rv[u], bf);
#pragma unroll
          for (int k = 0; k < VEC; ++k) one(lf[k], bf[k], k, of[k], inf[k]);
          st_stream(out + off, Vec16<TA>::pack(of));
          if constexpr (kInner) st_stream(inner + off, Vec16<TA>::pack(inf));
        }
      }
    } else {
      float lf[U], bf[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t rr = r + u * rstep;
        if (rr < rows) {
          lf[u] = to_f32(lora[rr * cols + vc]);
          bf[u] = to_f32(base[rr * cols + vc]);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t rr = r + u * rstep;
        if (rr < rows) {
          float o, in;
          one(lf[u], bf[u], 0, o, in);
          out[rr * cols + vc] = from_f32<TA>(o);
          if constexpr (kInner) inner[rr * cols + vc] = from_f32<TA>(in);
        }
      }
    }
  }
}

template <typename TA, typename TG, int V, bool kOutput, bool kBias>
static void launch_compose_v(const EwShape& sh, bool with_inner, bool inplace, const void* lora, const void* base,
                             const void* g, const void* bias, float s, void* out, void* inner, int64_t rows,
                             int64_t vcols, cudaStream_t st) {
  auto L = static_cast<const TA*>(lora);
  auto B = static_cast<const TA*>(base);
  auto G = static_cast<const TG*>(g);
  auto Bi = static_cast<const TA*>(bias);
  auto O = static_cast<TA*>(out);
  auto I = static_cast<TA*>(inner);
  if (with_inner)
    compose_fwd_kernel<TA, TG, V, true, true, kOutput, kBias><<<sh.grid, sh.block, 0, st>>>(L, B, G, Bi, s, O, I,
                                                                                          rows, vcols);
  else if (inplace || V == 1)
    compose_fwd_kernel<TA, TG, V, false, false, kOutput, kBias><<<sh.grid, sh.block, 0, st>>>(L, B, G, Bi, s, O,
                                                                                           I, rows, vcols);
  else
    compose_fwd_kernel<TA, TG, V, false, true, kOutput, kBias><<<sh.grid, sh.block, 0, st>>>(L, B, G, Bi, s, O, I,
                                                                                          rows, vcols);
}

template <typename TA, typename TG>
static int launch_compose(const void* lora, const void* base, const void* g, const void* bias, bool output_form,
                          float s, void* out, void* inner, int64_t rows, int64_t cols, cudaStream_t st) {
  constexpr int V = 16 / sizeof(TA);
  const bool vec = (cols % V == 0) && aligned16(lora) && aligned16(base) && aligned16(out) &&
                   (inner == nullptr || aligned16(inner));
  const int64_t vcols = vec ? cols / V : cols;
  if (vcols > int64_t(65535) * 64) return DORA_ERR_UNSUPPORTED;
  // A deep grid with streaming stores: up to 64 CTAs per SM's worth, but each thread
  // keeps at least three groups of four rows, and never fewer CTAs than 8 per SM's
  // worth.  Same GPU, layer-output form: 16384 x 28672 0.612 (8 per SM) / 0.589 (16) /
  // 0.570 ms (64); 8192 x 8192 0.0904 / 0.0894 / 0.0959 ms (64 leaves each thread less
  // than one group of rows).
  EwShape sh = ew_shape_deep(rows, vcols);
  const bool with_inner = inner != nullptr;
  const bool inplace = (out == lora);
#define DORA_COMPOSE_LAUNCH(VV)                                                                                     \
  do {                                                                                                              \
    if (!output_form)                                                                                               \
      launch_compose_v<TA, TG, VV, false, false>(sh, with_inner, inplace, lora, base, g, bias, s, out, inner, rows, \
                                                 vcols, st);                                                        \
    else if (bias)                                                                                                  \
      launch_compose_v<TA, TG, VV, true, true>(sh, with_inner, inplace, lora, base, g, bias, s, out, inner, rows,   \
                                               vcols, st);                                                          \
    else                                                                                                            \
      launch_compose_v<TA, TG, VV, true, false>(sh, with_inner, inplace, lora, base, g, bias, s, out, inner, rows,  \
                                                vcols, st);                                                         \
  } while (0)
  if (vec) DORA_COMPOSE_LAUNCH(V);
  else DORA_COMPOSE_LAUNCH(1);
#undef DORA_COMPOSE_LAUNCH
  return check_launch();
}

static bool ranges_overlap(const void* a, const void* b, size_t bytes) {
  auto x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + bytes && y < x + bytes;
}

static int compose_entry(const void* lora, const void* base, const void* bias, const void* g, int g_dtype,
                         double scale, void* out, void* inner, int64_t rows, int64_t cols, int act_dtype,
                         bool output_form, void* stream) {
  if (rows < 0 || cols < 0 || !dtype_ok(act_dtype) || !dtype_ok(g_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0) return DORA_OK;
  if (!lora || !base || !g || !out) return DORA_ERR_INVALID_ARGUMENT;
  const size_t bytes = size_t(rows) * size_t(cols) * dtype_size(act_dtype);
  if (inner && (ranges_overlap(inner, lora, bytes) || ranges_overlap(inner, base, bytes) ||
                ranges_overlap(inner, out, bytes)))
    return DORA_ERR_INVALID_ARGUMENT;
  if (inner && out == lora) return DORA_ERR_INVALID_ARGUMENT;  // the training form is out-of-place
  if (out != lora && ranges_overlap(out, lora, bytes)) return DORA_ERR_INVALID_ARGUMENT;
  if (ranges_overlap(out, base, bytes)) return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float s = float(scale);
  switch (act_dtype) {
    case DORA_DTYPE_BF16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_compose<__nv_bfloat16, float>(lora, base, g, bias, output_form, s, out, inner, rows, cols,
                                                        st)
                 : launch_compose<__nv_bfloat16, __nv_bfloat16>(lora, base, g, bias, output_form, s, out, inner, rows,
                                                                cols, st);
    case DORA_DTYPE_F16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_compose<__half, float>(lora, base, g, bias, output_form, s, out, inner, rows, cols, st)
                 : launch_compose<__half, __half>(lora, base, g, bias, output_form, s, out, inner, rows, cols, st);
    default:
      return launch_compose<float, float>(lora, base, g, bias, output_form, s, out, inner, rows, cols, st);
  }
}

}  // namespace dora

using namespace dora;

extern "C" int dora_compose_fwd(const void* lora, const void* base, const void* g, int g_dtype, double scale,
                                void* out, void* inner, int64_t rows, int64_t cols, int act_dtype,
                                void* stream) {
  return compose_entry(lora, base, nullptr, g, g_dtype, scale, out, inner, rows, cols, act_dtype, false, stream);
}

extern "C" int dora_linear_output_fwd(const void* lora, const void* result, const void* bias, const void* g,
                                      int g_dtype, double scale, void* y, void* inner, int64_t rows, int64_t cols,
                                      int act_dtype, void* stream) {
  return compose_entry(lora, result, bias, g, g_dtype, scale, y, inner, rows, cols, act_dtype, true, stream);
}
