// Internal interfaces shared by the factored-norm translation units.
#pragma once

#include "dora_common.cuh"

namespace dora {

enum { kGemmRowdot = 0, kGemmStore = 1 };

// CUDA-core kernels (norm_simt.cu).
template <int MODE, bool SSQ>
void simt_gemm(int dx, int dy, int dz, const void* X, int64_t ldx, const void* Y, int64_t ldy, const void* Z,
               int64_t ldz, int64_t M, int64_t N, int64_t K, int ksplit, float* rowdot, float* sumsq, float* C,
               int64_t ldc, cudaStream_t st);
void launch_row_sumsq(int dx, const void* X, int64_t M, int64_t K, float* out, cudaStream_t st);
// fp32 -> half (bf16 / fp16) copy, round to nearest even.
void launch_cast_to_half(const float* src, void* dst, int64_t n, int half_dtype, cudaStream_t st);
// tri_tile > 0: the partials hold only the tiles (i <= j) of tri_tile x tri_tile
// blocks; the lower blocks are read from their mirror images (G is symmetric).
void launch_gram_reduce(const float* part, int nsplit, int64_t r, float* yt, int half_dtype, void* hi, void* lo,
                        int tri_tile, cudaStream_t st);
void launch_norm_finalize(const float* wpart, int nw, const float* cpart, int nc, const float* bpart, int nb,
                          int64_t M, double scale, int out_dtype, void* norm_out, float* parts, cudaStream_t st);
// Low-rank finalize: G = sum of ng partial 16 x 16 Grams (fixed order), B G B^T per row
// on CUDA cores (r <= 16, B [M x r] in b_dtype), the slot sums and the assembly.
void launch_norm_finalize_gram(const float* wpart, int nw, const float* cpart, int nc, const float* gpart, int ng,
                               int r, const void* B, int b_dtype, int64_t M, double scale, int out_dtype,
                               void* norm_out, float* parts, cudaStream_t st);

// Tensor-core row-dot GEMM (norm_tc.cu).
struct TcGemmArgs {
  int dtype;                 // DORA_DTYPE_BF16 or DORA_DTYPE_F16 (X, Y1, Y2 and Z share it)
  const void* X;             // [M x K] row-major, ld = K
  const void* Y1;            // [N x K] row-major, ld = K
  const void* Y2;            // optional second Y, same shape; its k-blocks follow Y1's (X is re-read)
  const void* Z;             // rowdot mode: [M x N] row-major, ld = ldz
  int64_t ldz;
  int64_t M, N, K;
  int mode;                  // kGemmRowdot or kGemmStore
  bool sumsq;                // also emit sum_k X[m,k]^2 (rowdot mode, n-tile 0 only)
  int k_splits;              // contiguous K ranges per (m, n) tile
  float* rowdot_part;        // [n_tiles * k_splits][M]
  float* sumsq_part;         // [k_splits][M]
  float* C;                  // store mode: [k_splits][M][N] fp32
  // Fused B G B^T phase (rowdot mode, N <= 384): with G1 / G2 = the hi / lo halves of
  // G^T ([N x N] row-major), every split also adds rowsum(Z * (Z G^T)) over its share
  // of G's k-blocks into v_part[ks][M].  Requires tc_can_fuse_v(M, N, K).
  const void* G1 = nullptr;
  const void* G2 = nullptr;
  float* v_part = nullptr;
  // Store mode, M == N, symmetric product (the Gram matrix): 128 x 128 tiles and only
  // those with n_tile >= m_tile are computed; C's other tiles are left unwritten.
  bool tri = false;
  // Stream-K kernel, N tile of 16 without the fused B G B^T phase: also emit partial
  // Gram matrices A A^T, [grid][16 x 16] fp32 (one per CTA, fixed-order summable).
  float* g_part = nullptr;
  // Launch as an ordinary stream-ordered kernel instead of a programmatic dependent of
  // the previous launch (the kernel then needs no griddepcontrol.wait before reading
  // what earlier kernels wrote).
  bool plain_launch = false;
};
constexpr int kGramTile = 128;
struct TcGemmShape {
  int nt;        // N tile (columns of TMEM used)
  int n_tiles;
  int m_tiles;
  int kblocks;   // 64-wide k-blocks per Y operand
};
TcGemmShape tc_gemm_shape(int64_t M, int64_t N, int64_t K, int force_nt = 0);
bool tc_gemm_supported(int dtype, int64_t M, int64_t N, int64_t K, const void* X, const void* Y, const void* Z,
                       int64_t ldz);
int tc_rowdot_gemm(const TcGemmArgs& a, cudaStream_t st);
bool tc_can_fuse_v(int64_t M, int64_t N, int64_t K);

// CTA-pair row-dot GEMM (norm_tc2.cu): rowdot mode only, Z row stride 16-byte
// aligned, M >= 256, N tile <= 512.  Units are pairs of 128-row tiles.
bool tc2_supported(const TcGemmArgs& a);
int tc2_pairs(int64_t M);
int tc2_rowdot_gemm(const TcGemmArgs& a, cudaStream_t st);

// Stream-K row-dot kernel (norm_sk.cu): rowdot mode with the ||X||^2 row sums, one
// N tile (N <= 512), Z row stride 16-byte aligned, no Y2; optionally the fused
// B G B^T phase (G1 / G2 / v_part, tc_can_fuse_v).  The units of all tiles are
// split evenly over `grid` CTAs; partial slot s of a row comes from the s-th CTA
// that touches its tile, so rowdot_part, sumsq_part and v_part are [slots][M].
struct SkPlan {
  int grid, slots;
  int64_t units_per_tile, total_units;
};
bool tc_sk_supported(const TcGemmArgs& a);
SkPlan tc_sk_plan(int64_t M, int64_t N, int64_t K, bool fuse_v, int sms);
int tc_sk_rowdot_gemm(const TcGemmArgs& a, const SkPlan& p, cudaStream_t st);

// Stream-K row-dot kernel on CTA pairs (norm_sk2.cu): the same contract over
// 256-row pair tiles (M >= 256); SkPlan.grid counts clusters of two CTAs.
// N tiling of the CTA-pair stream-K kernel: the whole row up to 512 columns, the
// widest equal tiles of at most 512 columns above (unless overridden for comparison).
TcGemmShape tc2_sk_shape(int64_t M, int64_t N, int64_t K);
bool tc2_sk_supported(const TcGemmArgs& a);
SkPlan tc2_sk_plan(int64_t M, int64_t N, int64_t K, bool fuse_v, int sms, bool two_y = false);
int tc2_sk_rowdot_gemm(const TcGemmArgs& a, const SkPlan& p, cudaStream_t st);

}  // namespace dora
