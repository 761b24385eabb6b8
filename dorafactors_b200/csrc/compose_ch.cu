// DoRA compose forward / backward for convolution outputs: activations laid out
// [batch, channels, spatial...] (NCHW-style, contiguous) with g broadcast along the
// channel dimension, the layout _DoraConvNdLayer.forward composes
// (code/peft_patched/src/peft/tuners/lora/dora.py:1670-1715, g shaped
// [1, C, 1, ...]).  The reference runs this case on its eager PyTorch path (its
// fused kernels need g on the last dimension, dora_fused.py:563-574); the
// arithmetic here is the same per element as the linear kernels (compose.cu,
// backward.cu): fp32, one rounding per output, the reference's operand order.
//
// A "plane" is one (batch, channel) pair: `spatial` contiguous elements sharing
// one g.  Threads walk 16-byte chunks of a plane, so g is read once per plane.
//
// Backward column sum d_g[c] = sum over batch and spatial of inner * d_out,
// deterministic: CTA (c, z) folds batch split z of channel c in a fixed order,
// writes one partial, and the last CTA of the channel (completion counter, no
// spin-wait) adds the partials in split order and resets the counter.
#include "dora_common.cuh"

namespace dora {

template <typename TA, typename TG, int VEC, bool kInner>
__global__ void __launch_bounds__(256)
compose_ch_fwd_kernel(const TA* __restrict__ lora, const TA* __restrict__ base, const TG* __restrict__ g, float s,
                      TA* __restrict__ out, TA* __restrict__ inner, int64_t planes, int64_t channels,
                      int64_t vsp) {
  const int64_t sp = vsp * VEC;
  for (int64_t p = int64_t(blockIdx.y) * blockDim.y + threadIdx.y; p < planes; p += int64_t(gridDim.y) * blockDim.y) {
    const float gv = to_f32(g[p % channels]);
    const float gm1 = __fsub_rn(gv, 1.0f);
    for (int64_t v = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; v < vsp; v += int64_t(gridDim.x) * blockDim.x) {
      const int64_t off = p * sp + v * VEC;
      if constexpr (VEC > 1) {
        float lf[VEC], bf[VEC], of[VEC], inf[VEC];
        Vec16<TA>::unpack(ld_stream(lora + off), lf);
        Vec16<TA>::unpack(ld_stream(base + off), bf);
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          const float sl = __fmul_rn(s, lf[k]);
          of[k] = __fadd_rn(__fmul_rn(gm1, bf[k]), __fmul_rn(gv, sl));
          inf[k] = __fadd_rn(sl, bf[k]);
        }
        st_global(out + off, Vec16<TA>::pack(of));
        if constexpr (kInner) st_global(inner + off, Vec16<TA>::pack(inf));
      } else {
        const float l = to_f32(lora[off]), b = to_f32(base[off]);
        const float sl = __fmul_rn(s, l);
        out[off] = from_f32<TA>(__fadd_rn(__fmul_rn(gm1, b), __fmul_rn(gv, sl)));
        if constexpr (kInner) inner[off] = from_f32<TA>(__fadd_rn(sl, b));
      }
    }
  }
}

template <typename TA, typename TG, int VEC, bool kDL, bool kDB, bool kDG>
__global__ void __launch_bounds__(256)
compose_ch_bwd_kernel(const TA* __restrict__ d_out, const TA* __restrict__ inner, const TG* __restrict__ g, float s,
                      TA* __restrict__ d_lora, TA* __restrict__ d_base, TG* __restrict__ d_g,
                      unsigned* __restrict__ counters, float* __restrict__ partials, int64_t batch, int64_t channels,
                      int64_t vsp) {
  __shared__ float red[256];
  __shared__ bool is_last;
  const int64_t c = blockIdx.x;
  const int z = blockIdx.y, Z = gridDim.y;
  const int64_t n0 = batch * z / Z, n1 = batch * (z + 1) / Z;
  const int64_t sp = vsp * VEC;
  const float gv = to_f32(g[c]);
  const float gs = __fmul_rn(gv, s), gm1 = __fsub_rn(gv, 1.0f);
  float acc = 0.f;
  for (int64_t n = n0; n < n1; ++n) {
    const int64_t pbase = (n * channels + c) * sp;
    for (int64_t v = threadIdx.x; v < vsp; v += blockDim.x) {
      const int64_t off = pbase + v * VEC;
      if constexpr (VEC > 1) {
        float df[VEC], xf[VEC], lf[VEC], bf[VEC];
        Vec16<TA>::unpack(ld_stream(d_out + off), df);
        if constexpr (kDG) Vec16<TA>::unpack(ld_stream(inner + off), xf);
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          if constexpr (kDL) lf[k] = __fmul_rn(gs, df[k]);
          if constexpr (kDB) bf[k] = __fmul_rn(gm1, df[k]);
          if constexpr (kDG) acc = fmaf(xf[k], df[k], acc);
        }
        if constexpr (kDL) st_global(d_lora + off, Vec16<TA>::pack(lf));
        if constexpr (kDB) st_global(d_base + off, Vec16<TA>::pack(bf));
      } else {
        const float d = to_f32(d_out[off]);
        if constexpr (kDL) d_lora[off] = from_f32<TA>(__fmul_rn(gs, d));
        if constexpr (kDB) d_base[off] = from_f32<TA>(__fmul_rn(gm1, d));
        if constexpr (kDG) acc = fmaf(to_f32(inner[off]), d, acc);
      }
    }
  }
  if constexpr (kDG) {
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {  // fixed-shape tree
      if (int(threadIdx.x) < w) red[threadIdx.x] += red[threadIdx.x + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      partials[int64_t(z) * channels + c] = red[0];
      __threadfence();
      const unsigned done = atomicAdd(&counters[c], 1u);
      is_last = (done == unsigned(Z) - 1);
    }
    __syncthreads();
    if (is_last && threadIdx.x == 0) {
      __threadfence();
      float t = 0.f;
      for (int q = 0; q < Z; ++q) t += __ldcg(partials + int64_t(q) * channels + c);
      d_g[c] = from_f32<TG>(t);
      counters[c] = 0u;  // ready for the next call
    }
  }
}

// Launch shapes.
static dim3 ch_fwd_grid(int64_t planes, int64_t vsp, dim3& block) {
  int tx = 32;
  while (tx < 256 && tx < vsp) tx *= 2;
  block = dim3(unsigned(tx), unsigned(256 / tx), 1);
  const int64_t gx = (vsp + tx - 1) / tx;
  const int64_t target = int64_t(num_sms()) * 8;
  int64_t gy = (target + gx - 1) / gx;
  const int64_t need = (planes + block.y - 1) / block.y;
  if (gy > need) gy = need;
  if (gy < 1) gy = 1;
  if (gy > 65535) gy = 65535;
  return dim3(unsigned(gx > 65535 ? 65535 : gx), unsigned(gy), 1);
}
static int ch_bwd_splits(int64_t batch, int64_t channels) {
  int64_t z = (int64_t(num_sms()) * 4 + channels - 1) / (channels > 0 ? channels : 1);
  if (z > batch) z = batch;
  if (z > 1024) z = 1024;
  return int(z < 1 ? 1 : z);
}
static size_t ch_counter_bytes(int64_t channels) { return ((size_t(channels) * 4 + 255) / 256) * 256; }

template <typename TA, typename TG>
static int launch_ch_fwd(const void* lora, const void* base, const void* g, float s, void* out, void* inner,
                         int64_t batch, int64_t channels, int64_t spatial, cudaStream_t st) {
  constexpr int V = 16 / sizeof(TA);
  const bool vec = spatial % V == 0 && aligned16(lora) && aligned16(base) && aligned16(out) &&
                   (!inner || aligned16(inner));
  const int64_t vsp = vec ? spatial / V : spatial;
  const int64_t planes = batch * channels;
  dim3 block;
  const dim3 grid = ch_fwd_grid(planes, vsp, block);
  auto L = static_cast<const TA*>(lora);
  auto B = static_cast<const TA*>(base);
  auto G = static_cast<const TG*>(g);
  auto O = static_cast<TA*>(out);
  auto I = static_cast<TA*>(inner);
  if (vec) {
    if (inner) compose_ch_fwd_kernel<TA, TG, V, true><<<grid, block, 0, st>>>(L, B, G, s, O, I, planes, channels, vsp);
    else compose_ch_fwd_kernel<TA, TG, V, false><<<grid, block, 0, st>>>(L, B, G, s, O, I, planes, channels, vsp);
  } else {
    if (inner) compose_ch_fwd_kernel<TA, TG, 1, true><<<grid, block, 0, st>>>(L, B, G, s, O, I, planes, channels, vsp);
    else compose_ch_fwd_kernel<TA, TG, 1, false><<<grid, block, 0, st>>>(L, B, G, s, O, I, planes, channels, vsp);
  }
  return check_launch();
}

template <typename TA, typename TG, int V, bool DL, bool DB, bool DG>
static void launch_ch_bwd_v(dim3 grid, const void* d_out, const void* inner, const void* g, float s, void* d_lora,
                            void* d_base, void* d_g, unsigned* cnt, float* part, int64_t batch, int64_t channels,
                            int64_t vsp, cudaStream_t st) {
  compose_ch_bwd_kernel<TA, TG, V, DL, DB, DG><<<grid, 256, 0, st>>>(
      static_cast<const TA*>(d_out), static_cast<const TA*>(inner), static_cast<const TG*>(g), s,
      static_cast<TA*>(d_lora), static_cast<TA*>(d_base), static_cast<TG*>(d_g), cnt, part, batch, channels, vsp);
}

template <typename TA, typename TG, int V>
static void launch_ch_bwd_sel(dim3 grid, const void* d_out, const void* inner, const void* g, float s, void* d_lora,
                              void* d_base, void* d_g, unsigned* cnt, float* part, int64_t batch, int64_t channels,
                              int64_t vsp, cudaStream_t st) {
  const int sel = (d_lora ? 4 : 0) | (d_base ? 2 : 0) | (d_g ? 1 : 0);
#define DORA_CH_CASE(n, a, b, c)                                                                                   \
  case n:                                                                                                          \
    launch_ch_bwd_v<TA, TG, V, a, b, c>(grid, d_out, inner, g, s, d_lora, d_base, d_g, cnt, part, batch, channels, \
                                        vsp, st);                                                                  \
    break;
  switch (sel) {
    DORA_CH_CASE(1, false, false, true)
    DORA_CH_CASE(2, false, true, false)
    DORA_CH_CASE(3, false, true, true)
    DORA_CH_CASE(4, true, false, false)
    DORA_CH_CASE(5, true, false, true)
    DORA_CH_CASE(6, true, true, false)
    DORA_CH_CASE(7, true, true, true)
    default: break;
  }
#undef DORA_CH_CASE
}

template <typename TA, typename TG>
static int launch_ch_bwd(const void* d_out, const void* inner, const void* g, float s, void* d_lora, void* d_base,
                         void* d_g, void* ws, size_t ws_bytes, int64_t batch, int64_t channels, int64_t spatial,
                         cudaStream_t st) {
  constexpr int V = 16 / sizeof(TA);
  const bool vec = spatial % V == 0 && aligned16(d_out) && (!inner || aligned16(inner)) &&
                   (!d_lora || aligned16(d_lora)) && (!d_base || aligned16(d_base));
  const int64_t vsp = vec ? spatial / V : spatial;
  const int Z = ch_bwd_splits(batch, channels);
  unsigned* cnt = nullptr;
  float* part = nullptr;
  if (d_g) {
    const size_t need = ch_counter_bytes(channels) + size_t(Z) * size_t(channels) * 4;
    if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return DORA_ERR_WORKSPACE;
    cnt = static_cast<unsigned*>(ws);
    part = reinterpret_cast<float*>(static_cast<char*>(ws) + ch_counter_bytes(channels));
  }
  const dim3 grid(unsigned(channels), unsigned(Z), 1);
  if (vec) launch_ch_bwd_sel<TA, TG, V>(grid, d_out, inner, g, s, d_lora, d_base, d_g, cnt, part, batch, channels, vsp, st);
  else launch_ch_bwd_sel<TA, TG, 1>(grid, d_out, inner, g, s, d_lora, d_base, d_g, cnt, part, batch, channels, vsp, st);
  return check_launch();
}

static bool ch_shape_ok(int64_t batch, int64_t channels, int64_t spatial) {
  return batch >= 0 && channels >= 0 && spatial >= 0 && channels <= 2147483647 && batch <= (int64_t(1) << 40);
}

}  // namespace dora

using namespace dora;

extern "C" int dora_compose_fwd_channels(const void* lora, const void* base, const void* g, int g_dtype,
                                         double scale, void* out, void* inner, int64_t batch, int64_t channels,
                                         int64_t spatial, int act_dtype, void* stream) {
  if (!ch_shape_ok(batch, channels, spatial) || !dtype_ok(act_dtype) || !dtype_ok(g_dtype))
    return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (batch == 0 || channels == 0 || spatial == 0) return DORA_OK;
  // Out of place only (lora is read through the non-coherent path).
  if (!lora || !base || !g || !out || out == base || out == lora ||
      (inner && (inner == lora || inner == base || inner == out)))
    return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float s = float(scale);
  switch (act_dtype) {
    case DORA_DTYPE_BF16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_ch_fwd<__nv_bfloat16, float>(lora, base, g, s, out, inner, batch, channels, spatial, st)
                 : launch_ch_fwd<__nv_bfloat16, __nv_bfloat16>(lora, base, g, s, out, inner, batch, channels, spatial,
                                                               st);
    case DORA_DTYPE_F16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_ch_fwd<__half, float>(lora, base, g, s, out, inner, batch, channels, spatial, st)
                 : launch_ch_fwd<__half, __half>(lora, base, g, s, out, inner, batch, channels, spatial, st);
    default:
      return launch_ch_fwd<float, float>(lora, base, g, s, out, inner, batch, channels, spatial, st);
  }
}

extern "C" size_t dora_compose_bwd_channels_workspace_size(int64_t batch, int64_t channels, int64_t spatial,
                                                           int act_dtype) {
  if (!ch_shape_ok(batch, channels, spatial) || !dtype_ok(act_dtype) || channels == 0) return 0;
  (void)spatial;
  const int Z = ch_bwd_splits(batch > 0 ? batch : 1, channels);
  return ch_counter_bytes(channels) + size_t(Z) * size_t(channels) * 4;
}

extern "C" int dora_compose_bwd_channels(const void* d_out, const void* inner, const void* g, int g_dtype,
                                         double scale, void* d_lora, void* d_base, void* d_g, void* workspace,
                                         size_t workspace_bytes, int64_t batch, int64_t channels, int64_t spatial,
                                         int act_dtype, void* stream) {
  if (!ch_shape_ok(batch, channels, spatial) || !dtype_ok(act_dtype) || !dtype_ok(g_dtype))
    return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (!d_out || !g || (d_g && !inner)) return DORA_ERR_INVALID_ARGUMENT;
  if (channels == 0 || batch == 0) return DORA_OK;
  if (spatial == 0 && !d_g) return DORA_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float s = float(scale);
  switch (act_dtype) {
    case DORA_DTYPE_BF16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_ch_bwd<__nv_bfloat16, float>(d_out, inner, g, s, d_lora, d_base, d_g, workspace,
                                                       workspace_bytes, batch, channels, spatial, st)
                 : launch_ch_bwd<__nv_bfloat16, __nv_bfloat16>(d_out, inner, g, s, d_lora, d_base, d_g, workspace,
                                                               workspace_bytes, batch, channels, spatial, st);
    case DORA_DTYPE_F16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_ch_bwd<__half, float>(d_out, inner, g, s, d_lora, d_base, d_g, workspace, workspace_bytes,
                                                batch, channels, spatial, st)
                 : launch_ch_bwd<__half, __half>(d_out, inner, g, s, d_lora, d_base, d_g, workspace,
                                                 workspace_bytes, batch, channels, spatial, st);
    default:
      return launch_ch_bwd<float, float>(d_out, inner, g, s, d_lora, d_base, d_g, workspace, workspace_bytes, batch,
                                         channels, spatial, st);
  }
}
