// Row-sharded DoRA linear: the layer-output compose with the output all-gather
// fused in, for sm_100a.
//
// With out-features sharded over P ranks, rank p computes columns
// [col_offset, col_offset + cols) of y = result + delta, and every rank needs
// the whole [rows x ld] y.  Instead of composing into a local shard and then
// all-gathering it (one more pass over the shard, then a permute copy because
// the gathered shards arrive rank-major), this kernel stores each computed
// 16-byte vector of y straight into all P ranks' output buffers at its final
// position: the local one through HBM, the others through NVLink (peer
// pointers mapped into this process).  The NVLink traffic overlaps the
// compose's own HBM traffic, and y is written exactly once per rank.
//
// Per element the arithmetic is that of dora_linear_output_fwd (compose.cu):
//   base = result - bias, y = result + ((g - 1) * base + g * (s * lora)),
//   inner = s * lora + base (local, [rows x cols]),
// fp32 with one rounding per output and the reference's op order.
//
// Ordering with the peers is the caller's: every rank must be done reading
// the output buffers before any rank calls this, and must not read them until
// all ranks' calls have completed (a cross-rank barrier on the stream before
// and after).  With peers, each thread ends with a system-scope fence so its
// peer stores are performed before anything the stream runs next.
#include "dora_common.cuh"

namespace dora {

constexpr int kMaxRanks = 8;

struct RankPtrs {
  void* p[kMaxRanks];
};

// At most 128 registers: two 256-thread CTAs per SM, as the compose kernel.
template <typename TA, typename TG, int VEC, bool kInner, bool kBias>
__global__ void __launch_bounds__(256, 2)
compose_allgather_kernel(const TA* __restrict__ lora, const TA* __restrict__ result, const TG* __restrict__ g,
                         const TA* __restrict__ bias, float s, const __grid_constant__ RankPtrs y, int n_ranks,
                         int64_t col_offset,
                         int64_t ld, TA* __restrict__ inner, int64_t rows, int64_t vcols) {
  const int64_t vc = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vc < vcols) {
    const int64_t cols = vcols * VEC;
    float gv[VEC], gm1[VEC], bv[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      gv[k] = to_f32(g[vc * VEC + k]);
      gm1[k] = __fsub_rn(gv[k], 1.0f);
      bv[k] = kBias ? to_f32(bias[vc * VEC + k]) : 0.f;
    }
    const int64_t row0 = int64_t(blockIdx.y) * blockDim.y + threadIdx.y;
    const int64_t rstep = int64_t(gridDim.y) * blockDim.y;
    constexpr int U = 4;
    for (int64_t r = row0; r < rows; r += U * rstep) {
      if constexpr (VEC > 1) {
        uint4 lv[U], rv[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t rr = r + u * rstep;
          if (rr < rows) {
            const int64_t off = rr * cols + vc * VEC;
            lv[u] = ld_stream(lora + off);
            rv[u] = ld_stream(result + off);
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t rr = r + u * rstep;
          if (rr < rows) {
            float lf[VEC], rf[VEC], of[VEC], inf[VEC];
            Vec16<TA>::unpack(lv[u], lf);
            Vec16<TA>::unpack(rv[u], rf);
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
              const float b = kBias ? __fsub_rn(rf[k], bv[k]) : rf[k];
              const float sl = __fmul_rn(s, lf[k]);
              of[k] = __fadd_rn(rf[k], __fadd_rn(__fmul_rn(gm1[k], b), __fmul_rn(gv[k], sl)));
              if constexpr (kInner) inf[k] = __fadd_rn(sl, b);
            }
            const uint4 ov = Vec16<TA>::pack(of);
            const int64_t yoff = rr * ld + col_offset + vc * VEC;
            // The table is a __grid_constant__ parameter: indexed in place, not
            // copied to local memory, and read through the constant cache.
            for (int q = 0; q < n_ranks; ++q) st_global(static_cast<TA*>(y.p[q]) + yoff, ov);
            if constexpr (kInner) st_global(inner + rr * cols + vc * VEC, Vec16<TA>::pack(inf));
          }
        }
      } else {
        for (int64_t rr = r; rr < rows && rr < r + U * rstep; rr += rstep) {
          const float l = to_f32(lora[rr * cols + vc]);
          const float rv = to_f32(result[rr * cols + vc]);
          const float b = kBias ? __fsub_rn(rv, bv[0]) : rv;
          const float sl = __fmul_rn(s, l);
          const TA o = from_f32<TA>(__fadd_rn(rv, __fadd_rn(__fmul_rn(gm1[0], b), __fmul_rn(gv[0], sl))));
          const int64_t yoff = rr * ld + col_offset + vc;
          for (int q = 0; q < n_ranks; ++q) static_cast<TA*>(y.p[q])[yoff] = o;
          if constexpr (kInner) inner[rr * cols + vc] = from_f32<TA>(__fadd_rn(sl, b));
        }
      }
    }
  }
  // Peer stores are performed system-wide before this grid is seen to finish
  // (only when there are peers: with one rank every store is local).
  if (n_ranks > 1) __threadfence_system();
}

template <typename TA, typename TG, int V>
static void launch_allgather_v(const EwShape& sh, const void* lora, const void* result, const void* g,
                               const void* bias, float s, const RankPtrs& y, int n, int64_t col_offset,
                               int64_t ld, void* inner, int64_t rows, int64_t vcols, cudaStream_t st) {
  auto L = static_cast<const TA*>(lora);
  auto R = static_cast<const TA*>(result);
  auto G = static_cast<const TG*>(g);
  auto Bi = static_cast<const TA*>(bias);
  auto I = static_cast<TA*>(inner);
  if (inner && bias)
    compose_allgather_kernel<TA, TG, V, true, true><<<sh.grid, sh.block, 0, st>>>(L, R, G, Bi, s, y, n,
                                                                                  col_offset, ld, I, rows, vcols);
  else if (inner)
    compose_allgather_kernel<TA, TG, V, true, false><<<sh.grid, sh.block, 0, st>>>(L, R, G, Bi, s, y, n,
                                                                                   col_offset, ld, I, rows, vcols);
  else if (bias)
    compose_allgather_kernel<TA, TG, V, false, true><<<sh.grid, sh.block, 0, st>>>(L, R, G, Bi, s, y, n,
                                                                                   col_offset, ld, I, rows, vcols);
  else
    compose_allgather_kernel<TA, TG, V, false, false><<<sh.grid, sh.block, 0, st>>>(L, R, G, Bi, s, y, n,
                                                                                    col_offset, ld, I, rows, vcols);
}

template <typename TA, typename TG>
static int launch_allgather(const void* lora, const void* result, const void* g, const void* bias, float s,
                            const RankPtrs& y, int n, int64_t col_offset, int64_t ld, void* inner,
                            int64_t rows, int64_t cols, cudaStream_t st) {
  constexpr int V = 16 / sizeof(TA);
  bool vec = (cols % V == 0) && (col_offset % V == 0) && (ld % V == 0) && aligned16(lora) && aligned16(result) &&
             (inner == nullptr || aligned16(inner));
  for (int p = 0; p < n; ++p) vec = vec && aligned16(y.p[p]);
  const int64_t vcols = vec ? cols / V : cols;
  if (vcols > int64_t(65535) * 64) return DORA_ERR_UNSUPPORTED;
  const EwShape sh = ew_shape(rows, vcols);
  if (vec) launch_allgather_v<TA, TG, V>(sh, lora, result, g, bias, s, y, n, col_offset, ld, inner, rows, vcols, st);
  else launch_allgather_v<TA, TG, 1>(sh, lora, result, g, bias, s, y, n, col_offset, ld, inner, rows, vcols, st);
  return check_launch();
}

}  // namespace dora

using namespace dora;

extern "C" int dora_linear_output_fwd_allgather(const void* lora, const void* result, const void* bias,
                                                const void* g, int g_dtype, double scale, void* const* y_ranks,
                                                int n_ranks, int rank, int64_t col_offset, int64_t ld, void* inner,
                                                int64_t rows, int64_t cols, int act_dtype, void* stream) {
  if (rows < 0 || cols < 0 || !dtype_ok(act_dtype) || !dtype_ok(g_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (g_dtype != act_dtype && g_dtype != DORA_DTYPE_F32) return DORA_ERR_INVALID_ARGUMENT;
  if (n_ranks < 1 || n_ranks > kMaxRanks || rank < 0 || rank >= n_ranks || !y_ranks) return DORA_ERR_INVALID_ARGUMENT;
  if (col_offset < 0 || ld < cols || col_offset > ld - cols) return DORA_ERR_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0) return DORA_OK;
  if (!lora || !result || !g) return DORA_ERR_INVALID_ARGUMENT;
  const size_t esz = dtype_size(act_dtype), shard_bytes = size_t(rows) * size_t(cols) * esz;
  const size_t out_bytes = size_t(rows) * size_t(ld) * esz;
  auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
    const auto x = reinterpret_cast<uintptr_t>(a), z = reinterpret_cast<uintptr_t>(b);
    return x < z + nb && z < x + na;
  };
  if (inner && (overlap(inner, shard_bytes, lora, shard_bytes) || overlap(inner, shard_bytes, result, shard_bytes)))
    return DORA_ERR_INVALID_ARGUMENT;
  if (y_ranks[rank] && (overlap(y_ranks[rank], out_bytes, lora, shard_bytes) ||
                        overlap(y_ranks[rank], out_bytes, result, shard_bytes) ||
                        (inner && overlap(y_ranks[rank], out_bytes, inner, shard_bytes))))
    return DORA_ERR_INVALID_ARGUMENT;
  // Peers first, starting with the next rank, the local buffer last: each rank
  // begins its stores on a different link.
  RankPtrs y{};
  for (int q = 0; q < n_ranks; ++q) {
    const int p = (rank + 1 + q) % n_ranks;
    if (!y_ranks[p]) return DORA_ERR_INVALID_ARGUMENT;
    y.p[q] = y_ranks[p];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float s = float(scale);
  switch (act_dtype) {
    case DORA_DTYPE_BF16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_allgather<__nv_bfloat16, float>(lora, result, g, bias, s, y, n_ranks, col_offset, ld,
                                                          inner, rows, cols, st)
                 : launch_allgather<__nv_bfloat16, __nv_bfloat16>(lora, result, g, bias, s, y, n_ranks,
                                                                  col_offset, ld, inner, rows, cols, st);
    case DORA_DTYPE_F16:
      return g_dtype == DORA_DTYPE_F32
                 ? launch_allgather<__half, float>(lora, result, g, bias, s, y, n_ranks, col_offset, ld, inner,
                                                   rows, cols, st)
                 : launch_allgather<__half, __half>(lora, result, g, bias, s, y, n_ranks, col_offset, ld, inner,
                                                    rows, cols, st);
    default:
      return launch_allgather<float, float>(lora, result, g, bias, s, y, n_ranks, col_offset, ld, inner, rows,
                                            cols, st);
  }
}
