// Factored DoRA row norm: CUDA-core (fp32 FMA) kernels and the shared
// reduction / assembly kernels.
//
// The factored norm (dora.py:1024-1153) is
//   ||W0 + s B A||^2_row = ||W0||^2 + 2 s rowsum(B * (W0 A^T)) + s^2 rowsum((B G) * B),
//   G = A A^T.
// Both row sums are linear in the GEMM result, so every GEMM here is a
// "row-dot GEMM": C = X Y^T is formed tile by tile on chip and immediately
// contracted with Z (= B) along the row, leaving one float per row per tile.
// Tiles along N and splits along K write separate partial vectors that the
// finalize kernel adds in a fixed order, so the result is deterministic and
// the [out x r] products never reach HBM.
//
// The tensor-core path (norm_tc.cu) replaces the GEMMs for bf16/fp16; this
// file serves fp32 weights, mixed weight/adapter dtypes and odd alignments.
#include "dora_common.cuh"
#include "norm_internal.cuh"

namespace dora {

// ---------------------------------------------------------------------------
// Row-dot / store GEMM on CUDA cores.  64x64 tile, BK = 16, 256 threads, each
// thread a 4x4 sub-tile at stride 16 (conflict-free shared-memory reads).
// grid = (ceil(N/64), ceil(M/64), ksplit).
// ---------------------------------------------------------------------------
template <typename TX, typename TY, typename TZ, int MODE, bool kSumSq>
__global__ void __launch_bounds__(256)
simt_rowdot_gemm(const TX* __restrict__ X, int64_t ldx, const TY* __restrict__ Y, int64_t ldy,
                 const TZ* __restrict__ Z, int64_t ldz, int64_t M, int64_t N, int64_t K, int64_t kchunk,
                 float* __restrict__ rowdot_part, float* __restrict__ sumsq_part, float* __restrict__ C,
                 int64_t ldc) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
  const int64_t kb = int64_t(blockIdx.z) * kchunk;
  const int64_t ke = (kb + kchunk < K) ? kb + kchunk : K;
  float acc[4][4] = {};
  float ssq = 0.f;
  const bool do_ssq = kSumSq && blockIdx.x == 0;
  for (int64_t k0 = kb; k0 < ke; k0 += BK) {
    {  // each thread loads 4 consecutive k of one row of X and of Y
      const int lr = t >> 2, lk = (t & 3) * 4;
      const int64_t xm = m0 + lr, yn = n0 + lr;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t k = k0 + lk + q;
        As[lk + q][lr] = (xm < M && k < ke) ? to_f32(X[xm * ldx + k]) : 0.f;
        Bs[lk + q][lr] = (yn < N && k < ke) ? to_f32(Y[yn * ldy + k]) : 0.f;
      }
    }
    __syncthreads();
    if (do_ssq && t < BM) {
#pragma unroll
      for (int k = 0; k < BK; ++k) ssq = fmaf(As[k][t], As[k][t], ssq);
    }
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
  if (do_ssq && t < BM && m0 + t < M) sumsq_part[int64_t(blockIdx.z) * M + m0 + t] = ssq;
  if constexpr (MODE == kGemmRowdot) {
    const int64_t p = int64_t(blockIdx.z) * gridDim.x + blockIdx.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + ty + 16 * i;
      float v = 0.f;
      if (m < M) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t n = n0 + tx + 16 * j;
          if (n < N) v = fmaf(acc[i][j], to_f32(Z[m * ldz + n]), v);
        }
      }
      // Lanes tx = 0..15 of one half-warp hold the same row.
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (tx == 0 && m < M) rowdot_part[p * M + m] = v;
    }
  } else {
    float* Cz = C + int64_t(blockIdx.z) * M * ldc;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + ty + 16 * i;
      if (m >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + tx + 16 * j;
        if (n < N) Cz[m * ldc + n] = acc[i][j];
      }
    }
  }
}

// Sum of squares of each row (scale == 0 short-cut, dora.py:1117-1129).
template <typename TX>
__global__ void row_sumsq_kernel(const TX* __restrict__ X, int64_t M, int64_t K, float* __restrict__ out) {
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float s = 0.f;
  for (int64_t k = lane; k < K; k += 32) {
    const float v = to_f32(X[row * K + k]);
    s = fmaf(v, v, s);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) out[row] = s;
}

// Gram reduction: G = sum_z Gpart[z]; writes Y = G^T in fp32 (for the
// CUDA-core B G product) and, when hi/lo are given, the two-term split
// Y = hi + lo with hi, lo in the half type TH (for the tensor-core product).
// 32 x 32 tiles: the split partials are read along their rows (coalesced), summed
// in split order, and written transposed through shared memory.
template <typename TH>
__global__ void gram_reduce_kernel(const float* __restrict__ part, int nsplit, int64_t r, float* __restrict__ yt,
                                   TH* __restrict__ hi, TH* __restrict__ lo, int tri_tile) {
  __shared__ float tile[32][33];
  pdl_trigger();
  pdl_wait();  // the Gram partials come from the previous kernel
  const int64_t bi = int64_t(blockIdx.y) * 32, bj = int64_t(blockIdx.x) * 32;
  // A block below the computed triangle is read from its mirror (bj, bi), which
  // then needs no transpose on the way out.
  const bool mirror = tri_tile > 0 && (bi / tri_tile) > (bj / tri_tile);
  const int64_t ri = mirror ? bj : bi, rj = mirror ? bi : bj;
  const int tx = threadIdx.x;
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    const int64_t i = ri + yy, j = rj + tx;  // partial element [i][j]
    float v = 0.f;
    if (i < r && j < r) {
      // Eight split partials in flight per thread; the additions keep split order.
      const float* p = part + i * r + j;
      const int64_t rr = r * r;
      int z = 0;
      for (; z + 8 <= nsplit; z += 8) {
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = p[int64_t(z + q) * rr];
#pragma unroll
        for (int q = 0; q < 8; ++q) v += t[q];
      }
      if (z < nsplit) {
        // The last (or only) batch also keeps its loads in flight together: at r = 1024
        // (four splits) a one-by-one tail made this kernel 27 us instead of a few.
        float t[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) t[q] = (z + q < nsplit) ? p[int64_t(z + q) * rr] : 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (z + q < nsplit) v += t[q];
      }
    }
    tile[yy][tx] = v;
  }
  __syncthreads();
  for (int yy = threadIdx.y; yy < 32; yy += blockDim.y) {
    const int64_t oi = bj + yy, oj = bi + tx;  // Y[oi][oj] = G[oj][oi]
    if (oi < r && oj < r) {
      const float v = mirror ? tile[yy][tx] : tile[tx][yy];
      const int64_t idx = oi * r + oj;
      yt[idx] = v;
      if (hi) {
        const TH h = from_f32<TH>(v);
        hi[idx] = h;
        lo[idx] = from_f32<TH>(v - to_f32(h));
      }
    }
  }
}

// norm[m] = sqrt(max(w + (2s) c + (s^2) b, 0)), four rounded fp32 ops in the
// reference order (dora_fused.py:917-934), then cast to the weight dtype.
__device__ __forceinline__ float assemble_one(float w, float c, float b, float two_s, float s2) {
  const float t1 = __fmul_rn(two_s, c);
  const float p = __fadd_rn(w, t1);
  const float t2 = __fmul_rn(s2, b);
  float n2 = __fadd_rn(p, t2);
  n2 = (n2 > 0.f) ? n2 : ((n2 != n2) ? n2 : 0.f);  // clamp_min(0), NaN kept
  return __fsqrt_rn(n2);
}

template <typename TO>
__global__ void norm_finalize_kernel(const float* __restrict__ wpart, int nw, const float* __restrict__ cpart,
                                     int nc, const float* __restrict__ bpart, int nb, int64_t M, float two_s,
                                     float s2, bool scale_zero, TO* __restrict__ norm_out,
                                     float* __restrict__ parts) {
  pdl_wait();  // the partials come from the previous kernel
  const int64_t m = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (m >= M) return;
  // The partials are loaded eight at a time before they are added (in slot order),
  // so this kernel, which runs after the stream-K kernel on the call's critical
  // path, pays about one load latency instead of one per slot.
  auto slot_sum = [&](const float* __restrict__ part, int n) {
    float t = 0.f;
    for (int i = 0; i < n; i += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = i + j < n ? part[int64_t(i + j) * M + m] : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (i + j < n) t += v[j];
    }
    return t;
  };
  const float w = slot_sum(wpart, nw), c = slot_sum(cpart, nc), b = slot_sum(bpart, nb);
  float n;
  if (scale_zero) {
    const float x = (w > 0.f) ? w : ((w != w) ? w : 0.f);
    n = __fsqrt_rn(x);
  } else {
    n = assemble_one(w, c, b, two_s, s2);
  }
  norm_out[m] = from_f32<TO>(n);
  if (parts) {
    parts[m] = w;
    parts[M + m] = c;
    parts[2 * M + m] = b;
  }
}

// Low-rank finalize (r <= 16): G = sum over the stream-K CTAs' partial Grams in CTA
// order (each CTA of this grid forms it in shared memory: 256 entries x ng partials),
// then per row ba = B_j G B_j^T in fp32 (t_a = sum_b G_ab B_jb, ba = sum_a B_ja t_a,
// the reference's rowsum((B @ G) * B), dora.py:1132-1134), the slot sums and the
// assembly.
template <typename TO, typename TB>
__global__ void __launch_bounds__(256) norm_finalize_gram_kernel(
    const float* __restrict__ wpart, int nw, const float* __restrict__ cpart, int nc,
    const float* __restrict__ gpart, int ng, int r, const TB* __restrict__ B, int64_t M, float two_s, float s2,
    TO* __restrict__ norm_out, float* __restrict__ parts) {
  __shared__ float G[16][17];
  const int64_t m = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool live = m < M;
  // B is an input of the layer, not of the previous kernel: read before the wait
  // (r is 8 or 16, rows of r * 2 bytes on 16-byte boundaries).
  float bj[16];
  {
    uint4 q[2] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
    if (live) {
      const uint4* bp = reinterpret_cast<const uint4*>(B + m * r);
      q[0] = __ldg(bp);
      if (r > 8) q[1] = __ldg(bp + 1);
    }
    const TB* h = reinterpret_cast<const TB*>(q);
#pragma unroll
    for (int k = 0; k < 16; ++k) bj[k] = k < r ? to_f32(h[k]) : 0.f;
  }
  pdl_wait();  // the partials come from the previous kernel
  // This row's slot partials, issued before the Gram sum so their latency overlaps it.
  float w = 0.f, c = 0.f;
  if (live) {
    for (int i = 0; i < nw; ++i) w += wpart[int64_t(i) * M + m];
    for (int i = 0; i < nc; ++i) c += cpart[int64_t(i) * M + m];
  }
  {
    // 256 threads, one Gram entry each, summed in CTA order.  Up to 64 loads are in
    // flight before their additions, so the partials' latency is paid ng / 64 times:
    // this sum is on the call's critical path, after the stream-K kernel.
    const int e = threadIdx.x;
    float t = 0.f;
    for (int i = 0; i < ng; i += 64) {
      float v[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) v[j] = i + j < ng ? gpart[int64_t(i + j) * 256 + e] : 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (i + j < ng) t += v[j];
    }
    G[e >> 4][e & 15] = t;
  }
  __syncthreads();
  if (!live) return;
  float b = 0.f;
#pragma unroll
  for (int x = 0; x < 16; ++x) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < 16; ++y) t = fmaf(G[x][y], bj[y], t);
    b = fmaf(bj[x], t, b);
  }
  const float n = assemble_one(w, c, b, two_s, s2);
  norm_out[m] = from_f32<TO>(n);
  if (parts) {
    parts[m] = w;
    parts[M + m] = c;
    parts[2 * M + m] = b;
  }
}

// get_weight_norm (dora.py:1012-1022): one warp per row.
template <typename TW, typename TL>
__global__ void dense_norm_kernel(const TW* __restrict__ W, const TL* __restrict__ L, float s, int64_t M, int64_t K,
                                  TW* __restrict__ out) {
  const int64_t row = int64_t(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float acc = 0.f;
  for (int64_t k = lane; k < K; k += 32) {
    const float t = __fadd_rn(to_f32(W[row * K + k]), __fmul_rn(s, to_f32(L[row * K + k])));
    acc = fmaf(t, t, acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) out[row] = from_f32<TW>(__fsqrt_rn(acc));
}

template <typename TW>
static void launch_dense_norm(int ld, const void* W, const void* L, float s, int64_t M, int64_t K, void* out,
                              cudaStream_t st) {
  const unsigned grid = unsigned((M + 7) / 8);
  auto w = static_cast<const TW*>(W);
  auto o = static_cast<TW*>(out);
  switch (ld) {
    case DORA_DTYPE_BF16: dense_norm_kernel<<<grid, 256, 0, st>>>(w, static_cast<const __nv_bfloat16*>(L), s, M, K, o); break;
    case DORA_DTYPE_F16: dense_norm_kernel<<<grid, 256, 0, st>>>(w, static_cast<const __half*>(L), s, M, K, o); break;
    default: dense_norm_kernel<<<grid, 256, 0, st>>>(w, static_cast<const float*>(L), s, M, K, o); break;
  }
}

__global__ void assembly_kernel(const float* __restrict__ w, const float* __restrict__ c, const float* __restrict__ b,
                                float two_s, float s2, float* __restrict__ out, int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = assemble_one(w[i], c[i], b[i], two_s, s2);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <typename TX, typename TY, typename TZ, int MODE, bool SSQ>
static void launch_simt(const void* X, int64_t ldx, const void* Y, int64_t ldy, const void* Z, int64_t ldz, int64_t M,
                        int64_t N, int64_t K, int ksplit, float* rowdot, float* ssq, float* C, int64_t ldc,
                        cudaStream_t st) {
  const int64_t kchunk = ((K + ksplit - 1) / ksplit + 15) / 16 * 16;
  dim3 grid(unsigned((N + 63) / 64), unsigned((M + 63) / 64), unsigned(ksplit));
  simt_rowdot_gemm<TX, TY, TZ, MODE, SSQ><<<grid, 256, 0, st>>>(
      static_cast<const TX*>(X), ldx, static_cast<const TY*>(Y), ldy, static_cast<const TZ*>(Z), ldz, M, N, K,
      kchunk, rowdot, ssq, C, ldc);
}

// Dispatch on three runtime dtypes.
template <int MODE, bool SSQ, typename TX, typename TY>
static void simt_z(int dz, const void* X, int64_t ldx, const void* Y, int64_t ldy, const void* Z, int64_t ldz,
                   int64_t M, int64_t N, int64_t K, int ks, float* rd, float* ss, float* C, int64_t ldc,
                   cudaStream_t st) {
  switch (dz) {
    case DORA_DTYPE_BF16: launch_simt<TX, TY, __nv_bfloat16, MODE, SSQ>(X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
    case DORA_DTYPE_F16: launch_simt<TX, TY, __half, MODE, SSQ>(X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
    default: launch_simt<TX, TY, float, MODE, SSQ>(X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
  }
}
template <int MODE, bool SSQ, typename TX>
static void simt_y(int dy, int dz, const void* X, int64_t ldx, const void* Y, int64_t ldy, const void* Z, int64_t ldz,
                   int64_t M, int64_t N, int64_t K, int ks, float* rd, float* ss, float* C, int64_t ldc,
                   cudaStream_t st) {
  switch (dy) {
    case DORA_DTYPE_BF16: simt_z<MODE, SSQ, TX, __nv_bfloat16>(dz, X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
    case DORA_DTYPE_F16: simt_z<MODE, SSQ, TX, __half>(dz, X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
    default: simt_z<MODE, SSQ, TX, float>(dz, X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
  }
}
template <int MODE, bool SSQ>
void simt_gemm(int dx, int dy, int dz, const void* X, int64_t ldx, const void* Y, int64_t ldy, const void* Z,
               int64_t ldz, int64_t M, int64_t N, int64_t K, int ks, float* rd, float* ss, float* C, int64_t ldc,
               cudaStream_t st) {
  switch (dx) {
    case DORA_DTYPE_BF16: simt_y<MODE, SSQ, __nv_bfloat16>(dy, dz, X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
    case DORA_DTYPE_F16: simt_y<MODE, SSQ, __half>(dy, dz, X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
    default: simt_y<MODE, SSQ, float>(dy, dz, X, ldx, Y, ldy, Z, ldz, M, N, K, ks, rd, ss, C, ldc, st); break;
  }
}
template void simt_gemm<kGemmRowdot, true>(int, int, int, const void*, int64_t, const void*, int64_t, const void*,
                                           int64_t, int64_t, int64_t, int64_t, int, float*, float*, float*, int64_t,
                                           cudaStream_t);
template void simt_gemm<kGemmRowdot, false>(int, int, int, const void*, int64_t, const void*, int64_t, const void*,
                                            int64_t, int64_t, int64_t, int64_t, int, float*, float*, float*, int64_t,
                                            cudaStream_t);
template void simt_gemm<kGemmStore, false>(int, int, int, const void*, int64_t, const void*, int64_t, const void*,
                                           int64_t, int64_t, int64_t, int64_t, int, float*, float*, float*, int64_t,
                                           cudaStream_t);

// fp32 -> bf16 / fp16, round to nearest even, four elements per thread and step.
template <typename TH>
__global__ void cast_to_half_kernel(const float* __restrict__ src, TH* __restrict__ dst, int64_t n, bool vec) {
  const int64_t n4 = vec ? n / 4 : 0;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(src) + i);
    TH h[4] = {from_f32<TH>(v.x), from_f32<TH>(v.y), from_f32<TH>(v.z), from_f32<TH>(v.w)};
    *reinterpret_cast<uint2*>(dst + 4 * i) = *reinterpret_cast<const uint2*>(h);
  }
  for (int64_t i = 4 * n4 + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = from_f32<TH>(src[i]);
}

void launch_cast_to_half(const float* src, void* dst, int64_t n, int half_dtype, cudaStream_t st) {
  const bool vec = aligned16(src) && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0;
  int64_t blocks = (n / 4 + 255) / 256;
  const int64_t cap = int64_t(num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (half_dtype == DORA_DTYPE_F16)
    cast_to_half_kernel<<<unsigned(blocks), 256, 0, st>>>(src, static_cast<__half*>(dst), n, vec);
  else
    cast_to_half_kernel<<<unsigned(blocks), 256, 0, st>>>(src, static_cast<__nv_bfloat16*>(dst), n, vec);
}

void launch_row_sumsq(int dx, const void* X, int64_t M, int64_t K, float* out, cudaStream_t st) {
  const unsigned grid = unsigned((M + 7) / 8);
  switch (dx) {
    case DORA_DTYPE_BF16: row_sumsq_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(X), M, K, out); break;
    case DORA_DTYPE_F16: row_sumsq_kernel<<<grid, 256, 0, st>>>(static_cast<const __half*>(X), M, K, out); break;
    default: row_sumsq_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(X), M, K, out); break;
  }
}

void launch_gram_reduce(const float* part, int nsplit, int64_t r, float* yt, int half_dtype, void* hi, void* lo,
                        int tri_tile, cudaStream_t st) {
  const unsigned nb = unsigned((r + 31) / 32);
  const dim3 grid(nb, nb), block(32, 32);
  cudaError_t e;
  if (half_dtype == DORA_DTYPE_F16)
    e = launch_pdl(gram_reduce_kernel<__half>, grid, block, 0, st, part, nsplit, r, yt, static_cast<__half*>(hi),
                   static_cast<__half*>(lo), tri_tile);
  else
    e = launch_pdl(gram_reduce_kernel<__nv_bfloat16>, grid, block, 0, st, part, nsplit, r, yt,
                   static_cast<__nv_bfloat16*>(hi), static_cast<__nv_bfloat16*>(lo), tri_tile);
  if (e != cudaSuccess) set_cuda_error(e);
}

void launch_norm_finalize(const float* wpart, int nw, const float* cpart, int nc, const float* bpart, int nb,
                          int64_t M, double scale, int out_dtype, void* norm_out, float* parts, cudaStream_t st) {
  const float two_s = float(2.0 * scale), s2 = float(scale * scale);
  const bool sz = (scale == 0.0);
  const dim3 grid(unsigned((M + 255) / 256)), block(256);
  cudaError_t e;
  switch (out_dtype) {
    case DORA_DTYPE_BF16:
      e = launch_pdl(norm_finalize_kernel<__nv_bfloat16>, grid, block, 0, st, wpart, nw, cpart, nc, bpart, nb, M,
                     two_s, s2, sz, static_cast<__nv_bfloat16*>(norm_out), parts);
      break;
    case DORA_DTYPE_F16:
      e = launch_pdl(norm_finalize_kernel<__half>, grid, block, 0, st, wpart, nw, cpart, nc, bpart, nb, M, two_s,
                     s2, sz, static_cast<__half*>(norm_out), parts);
      break;
    default:
      e = launch_pdl(norm_finalize_kernel<float>, grid, block, 0, st, wpart, nw, cpart, nc, bpart, nb, M, two_s,
                     s2, sz, static_cast<float*>(norm_out), parts);
      break;
  }
  if (e != cudaSuccess) set_cuda_error(e);
}

template <typename TO>
static cudaError_t launch_finalize_gram_t(const float* wpart, int nw, const float* cpart, int nc, const float* gpart,
                                          int ng, int r, const void* B, int b_dtype, int64_t M, float two_s, float s2,
                                          void* norm_out, float* parts, cudaStream_t st) {
  const dim3 grid(unsigned((M + 255) / 256)), block(256);
  if (b_dtype == DORA_DTYPE_F16)
    return launch_pdl(norm_finalize_gram_kernel<TO, __half>, grid, block, 0, st, wpart, nw, cpart, nc, gpart, ng, r,
                      static_cast<const __half*>(B), M, two_s, s2, static_cast<TO*>(norm_out), parts);
  return launch_pdl(norm_finalize_gram_kernel<TO, __nv_bfloat16>, grid, block, 0, st, wpart, nw, cpart, nc, gpart, ng,
                    r, static_cast<const __nv_bfloat16*>(B), M, two_s, s2, static_cast<TO*>(norm_out), parts);
}

void launch_norm_finalize_gram(const float* wpart, int nw, const float* cpart, int nc, const float* gpart, int ng,
                               int r, const void* B, int b_dtype, int64_t M, double scale, int out_dtype,
                               void* norm_out, float* parts, cudaStream_t st) {
  const float two_s = float(2.0 * scale), s2 = float(scale * scale);
  cudaError_t e;
  switch (out_dtype) {
    case DORA_DTYPE_F16:
      e = launch_finalize_gram_t<__half>(wpart, nw, cpart, nc, gpart, ng, r, B, b_dtype, M, two_s, s2, norm_out,
                                         parts, st);
      break;
    default:
      e = launch_finalize_gram_t<__nv_bfloat16>(wpart, nw, cpart, nc, gpart, ng, r, B, b_dtype, M, two_s, s2,
                                                norm_out, parts, st);
      break;
  }
  if (e != cudaSuccess) set_cuda_error(e);
}

}  // namespace dora

using namespace dora;

extern "C" int dora_norm_assembly(const float* w_norm_sq, const float* cross, const float* ba, double scale,
                                  float* norm_out, int64_t n, void* stream) {
  if (n < 0) return DORA_ERR_INVALID_ARGUMENT;
  if (n == 0) return DORA_OK;
  if (!w_norm_sq || !cross || !ba || !norm_out) return DORA_ERR_INVALID_ARGUMENT;
  // Coefficients formed in double and rounded to fp32, like PyTorch's
  // Python-scalar promotion (dora_fused.py:970-975).
  const float two_s = float(2.0 * scale), s2 = float(scale * scale);
  assembly_kernel<<<unsigned((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(w_norm_sq, cross, ba,
                                                                                            two_s, s2, norm_out, n);
  return check_launch();
}

extern "C" int dora_weight_norm_dense(const void* W, const void* L, int64_t out_features, int64_t in_features,
                                      int w_dtype, int l_dtype, double scale, void* norm_out, void* stream) {
  if (out_features < 0 || in_features < 0 || !dtype_ok(w_dtype) || !dtype_ok(l_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (out_features == 0) return DORA_OK;
  if (!norm_out || (in_features > 0 && (!W || !L))) return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float s = float(scale);
  switch (w_dtype) {
    case DORA_DTYPE_BF16: launch_dense_norm<__nv_bfloat16>(l_dtype, W, L, s, out_features, in_features, norm_out, st); break;
    case DORA_DTYPE_F16: launch_dense_norm<__half>(l_dtype, W, L, s, out_features, in_features, norm_out, st); break;
    default: launch_dense_norm<float>(l_dtype, W, L, s, out_features, in_features, norm_out, st); break;
  }
  return check_launch();
}
