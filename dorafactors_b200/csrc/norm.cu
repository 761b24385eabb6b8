// dora_weight_norm: plan, workspace layout and launch sequence of the
// factored row norm (dora.py:1024-1153).
//
// Launches (tensor-core path, bf16 weights and adapters):
//   1. Gram partials   G_z = A[:, Kz] A[:, Kz]^T       tcgen05, split-K, fp32 store
//   2. Gram reduce     G = sum_z G_z; Y = G^T as fp32 and as a bf16 hi + lo pair
//   3. cross term      rowsum(B * (W0 A^T)) and ||W0||^2   tcgen05 row-dot, stream-K
//                      (one CTA per SM, equal shares of all tiles' k-blocks)
//   4. B G B^T term    rowsum(B * (B Y_hi^T + B Y_lo^T))   tcgen05 row-dot; for r <= 384
//                      it runs inside launch 3, each split taking its share of
//                      G's k-blocks with the B tile already staged in shared memory
//   5. finalize        fixed-order partial sums + norm assembly + cast
// fp16 runs step 4 on CUDA cores from the fp32 G (an fp16 hi/lo split could
// overflow for large Gram entries).  The two-term split keeps about 16
// significant bits of G, so B G B^T carries a relative error near 2^-16
// instead of bf16's 2^-8.
//
// Half-precision weights with fp32 adapters (PEFT's default: adapters upcast to
// fp32 on a bf16 / fp16 base) first round the adapters into the weight dtype
// (step 0, copies in the workspace) and then take the tensor-core path: each
// adapter entry moves by at most half an ulp of the weight dtype, so the cross
// and B G B^T terms carry a relative error of about that size, below the
// rounding of the norm itself into the weight dtype.  fp32 weights run steps
// 1, 3 and 4 on CUDA cores in fp32.
#include <cstdlib>

#include "norm_internal.cuh"

namespace dora {

struct NormPlan {
  bool cast_a, cast_b;  // fp32 adapters rounded into the (half) weight dtype first
  bool tc_u, tc_v, tc_g, fuse_v, pair_u, sk_u, sk2_u;
  bool fuse_g;  // r <= 16: Gram inside the stream-K kernel, B G B^T in the finalize
  bool v_pair;  // B G B^T on the CTA-pair stream-K kernel: one launch for G's hi half, one for lo
  SkPlan sk, vsk;
  int gram_splits, u_splits, u_ntiles, v_splits, v_ntiles;
  size_t off_a, off_bh, off_gpart, off_yt, off_hi, off_lo, off_w, off_c, off_b, off_g16, off_vs, total;
};

static size_t up256(size_t x) { return (x + 255) / 256 * 256; }

// Choose a K split so that (tiles x splits) fills the GPU in close to whole
// waves; every split costs one extra epilogue, weighed at 2%.
static int pick_splits(int64_t tiles, int kb_total, int sms, int max_splits) {
  int best = 1;
  double best_score = -1.0;
  for (int s = 1; s <= max_splits && s <= kb_total; ++s) {
    const double units = double(tiles) * s;
    const double waves = double((int64_t(units) + sms - 1) / sms);
    const double score = (units / sms) / waves * (1.0 - 0.02 * (s - 1));
    if (score > best_score + 1e-9) {
      best_score = score;
      best = s;
    }
  }
  return best;
}

// DORA_B200_PAIR=1 selects the CTA-pair cross-term kernel.  The single-CTA
// kernel is the default: at 28672 x 8192, r = 384 it measured 0.248 ms against
// the pair's 0.257 ms once both issue their MMAs at the full tensor-pipe rate.
static bool use_pair_kernel() {
  static const bool on = [] {
    const char* e = std::getenv("DORA_B200_PAIR");
    return e && e[0] == '1';
  }();
  return on;
}

// The CTA-pair stream-K cross-term kernel runs for N tiles of 256 columns and more
// (r > 240), where halving the A-operand bytes per SM pays for the pair's longer
// slot hand-off (28672 x 8192: 0.205 vs 0.212 ms at r = 384; 8192 x 8192: 0.116 vs
// 0.134 ms at r = 512, 0.066 vs 0.058 ms at r = 16).  DORA_B200_SK2=1 / 0 forces it
// on / off.
static int sk2_mode() {
  static const int mode = [] {
    const char* e = std::getenv("DORA_B200_SK2");
    return e ? (e[0] == '1' ? 1 : 0) : -1;
  }();
  return mode;
}

// DORA_B200_FUSE_G=0 keeps the separate Gram launches at r <= 16.
static bool use_fused_gram() {
  static const bool on = [] {
    const char* e = std::getenv("DORA_B200_FUSE_G");
    return !(e && e[0] == '0');
  }();
  return on;
}

// DORA_B200_SK=0 selects the split-K cross-term kernel instead of the stream-K one.
static bool use_sk_kernel() {
  static const bool on = [] {
    const char* e = std::getenv("DORA_B200_SK");
    return !(e && e[0] == '0');
  }();
  return on;
}

// `aligned`: W (and A / B where they are used in place) start on 16 bytes.
static NormPlan make_plan(int64_t out, int64_t in, int64_t r, int wdt, int adt, int bdt, bool aligned) {
  NormPlan p{};
  const int sms = num_sms();
  const bool half_w = wdt == DORA_DTYPE_BF16 || wdt == DORA_DTYPE_F16;
  p.cast_a = half_w && adt == DORA_DTYPE_F32 && (bdt == DORA_DTYPE_F32 || bdt == wdt);
  p.cast_b = half_w && bdt == DORA_DTYPE_F32 && (adt == DORA_DTYPE_F32 || adt == wdt);
  if (p.cast_a) adt = wdt;
  if (p.cast_b) bdt = wdt;
  const bool half_uniform = (wdt == adt && adt == bdt) && half_w;
  p.tc_u = half_uniform && aligned && in % 8 == 0 && in > 0;
  p.tc_g = p.tc_u;
  p.tc_v = p.tc_u && wdt == DORA_DTYPE_BF16 && r % 8 == 0;
  // Gram partials
  if (p.tc_g) {
    // Symmetric: 128 x 128 tiles, upper triangle only.
    const TcGemmShape g = tc_gemm_shape(r, r, in, kGramTile);
    const int64_t tiles = int64_t(g.m_tiles) * (g.m_tiles + 1) / 2;
    int s = int(sms / (tiles > 0 ? tiles : 1));
    // At least 4 k-blocks per split: each split's partial tile is re-read by the reduce,
    // and a split much shorter than the pipeline depth only adds latency.
    const int per = 4;
    const int cap = g.kblocks / per > 0 ? g.kblocks / per : 1;
    p.gram_splits = s < 1 ? 1 : (s > cap ? cap : s);
  } else {
    const int64_t tiles = ((r + 63) / 64) * ((r + 63) / 64);
    const int64_t kb = (in + 255) / 256;
    int64_t s = (2 * sms) / (tiles > 0 ? tiles : 1);
    if (s > kb) s = kb;
    p.gram_splits = int(s < 1 ? 1 : s);
  }
  // Cross term: stream-K on CTA pairs (wide N tiles) or single CTAs; the split-K
  // kernels when neither applies (or when selected for comparison).
  p.fuse_v = p.tc_u && p.tc_v && tc_can_fuse_v(out, r, in);
  // Low rank (r <= 16, one 16-column N tile): the stream-K kernel's row warps also add
  // up the Gram matrix from the A tiles they already hold, and the finalize forms
  // B G B^T on CUDA cores (256 FMAs per row), so the Gram, its reduce and the
  // B G B^T units leave the launch sequence.
  p.fuse_g = p.tc_u && r <= 16 && r % 8 == 0 && use_fused_gram() && use_sk_kernel() && !use_pair_kernel() && sk2_mode() != 1;
  if (p.fuse_g) p.fuse_v = false;
  if (p.tc_u) {
    const TcGemmShape u = tc_gemm_shape(out, r, in);
    TcGemmArgs probe{};
    probe.mode = kGemmRowdot;
    probe.Z = reinterpret_cast<const void*>(uintptr_t(256));  // alignment is checked per call
    probe.ldz = r;
    probe.M = out;
    probe.N = r;
    probe.K = in;
    probe.sumsq = true;
    if (p.fuse_v) {
      probe.G1 = probe.Z;
      probe.G2 = probe.Z;
      probe.v_part = reinterpret_cast<float*>(uintptr_t(256));
    }
    p.pair_u = use_pair_kernel() && tc2_supported(probe);
    const int m2 = sk2_mode();
    const TcGemmShape u2 = tc2_sk_shape(out, r, in);
    if (p.fuse_v && u2.n_tiles > 1 && !p.pair_u && use_sk_kernel() && (m2 == 1 || (m2 < 0 && u.nt >= 256))) {
      // The pair kernel with several N tiles has no fused B G B^T phase.
      p.fuse_v = false;
      probe.G1 = probe.G2 = nullptr;
      probe.v_part = nullptr;
    }
    p.sk2_u = !p.pair_u && use_sk_kernel() && (m2 == 1 || (m2 < 0 && u.nt >= 256)) && tc2_sk_supported(probe);
    p.sk_u = !p.pair_u && !p.sk2_u && use_sk_kernel() && tc_sk_supported(probe);
    if (p.fuse_g && !p.sk_u) p.fuse_g = false;  // the single-CTA stream-K kernel carries the Gram
    p.u_ntiles = p.sk2_u ? u2.n_tiles : u.n_tiles;
    if (p.sk2_u) {
      p.sk = tc2_sk_plan(out, r, in, p.fuse_v, sms);
      p.u_splits = p.sk.slots;
    } else if (p.sk_u) {
      p.sk = tc_sk_plan(out, r, in, p.fuse_v, sms);
      p.u_splits = p.sk.slots;
    } else {
      p.u_splits = p.pair_u ? pick_splits(int64_t(tc2_pairs(out)) * u.n_tiles, u.kblocks, sms / 2, 8)
                            : pick_splits(int64_t(u.m_tiles) * u.n_tiles, u.kblocks, sms, 8);
    }
  } else {
    p.u_ntiles = int((r + 63) / 64);
    const int64_t tiles = ((out + 63) / 64) * p.u_ntiles;
    int64_t s = (4 * sms) / (tiles > 0 ? tiles : 1);
    const int64_t kb = (in + 255) / 256;
    if (s > kb) s = kb;
    p.u_splits = int(s < 1 ? 1 : s);
  }
  // B G B^T term: folded into the cross-term kernel when its tile fits, else its own launch.
  if (p.fuse_v) {
    p.v_ntiles = 1;
    p.v_splits = p.u_splits;
  } else if (p.tc_v) {
    // Above r = 512 the CTA-pair stream-K kernel forms B (G_hi + G_lo) in one launch (G_lo
    // as a second Y), X = Z = B, its ||B||^2 output to scratch (8192^2: r = 768 0.168 ->
    // 0.158 ms, r = 1024 0.212 -> 0.186 ms); at r = 512 the split-K launch is faster
    // (0.099-0.103 against 0.110 ms).
    TcGemmArgs vp{};
    vp.mode = kGemmRowdot;
    vp.Z = reinterpret_cast<const void*>(uintptr_t(256));
    vp.ldz = r;
    vp.M = out;
    vp.N = r;
    vp.K = r;
    vp.sumsq = true;
    vp.Y1 = vp.Y2 = vp.Z;
    p.v_pair = r > 512 && use_sk_kernel() && sk2_mode() != 0 && !use_pair_kernel() && tc2_sk_supported(vp);
    if (p.v_pair) {
      p.vsk = tc2_sk_plan(out, r, r, false, sms, true);
      p.v_splits = p.vsk.slots;
      p.v_ntiles = tc2_sk_shape(out, r, r).n_tiles;
    } else {
      const TcGemmShape v = tc_gemm_shape(out, r, r);
      p.v_ntiles = v.n_tiles;
      p.v_splits = pick_splits(int64_t(v.m_tiles) * v.n_tiles, 2 * v.kblocks, sms, 4);
    }
  } else {
    p.v_ntiles = int((r + 63) / 64);
    p.v_splits = 1;
  }
  size_t o = 0;
  p.off_a = o;     o += p.cast_a ? up256(size_t(r) * in * 2) : 0;
  p.off_bh = o;    o += p.cast_b ? up256(size_t(out) * r * 2) : 0;
  p.off_gpart = o; o += up256(size_t(p.gram_splits) * r * r * 4);
  p.off_yt = o;    o += up256(size_t(r) * r * 4);
  p.off_hi = o;    o += up256(size_t(r) * r * 2);
  p.off_lo = o;    o += up256(size_t(r) * r * 2);
  p.off_w = o;     o += up256(size_t(p.u_splits) * out * 4);
  p.off_c = o;     o += up256(size_t(p.u_splits) * p.u_ntiles * out * 4);
  p.off_b = o;     o += up256(size_t(p.v_splits) * p.v_ntiles * out * 4);
  p.off_g16 = o;   o += p.fuse_g ? up256(size_t(p.sk.grid) * 256 * 4) : 0;
  p.off_vs = o;    o += p.v_pair ? up256(size_t(p.vsk.slots) * out * 4) : 0;
  p.total = o;
  return p;
}

}  // namespace dora

using namespace dora;

extern "C" size_t dora_weight_norm_workspace_size(int64_t out_features, int64_t in_features, int64_t rank,
                                                  int w_dtype, int a_dtype, int b_dtype) {
  if (out_features <= 0 || in_features < 0 || rank < 0) return 0;
  if (!dtype_ok(w_dtype) || !dtype_ok(a_dtype) || !dtype_ok(b_dtype)) return 0;
  // The aligned plan is never smaller than the unaligned one for the same shape.
  NormPlan a = make_plan(out_features, in_features, rank, w_dtype, a_dtype, b_dtype, true);
  NormPlan b = make_plan(out_features, in_features, rank, w_dtype, a_dtype, b_dtype, false);
  return a.total > b.total ? a.total : b.total;
}

extern "C" int dora_weight_norm(const void* W, const void* A, const void* B, int64_t out_features,
                                int64_t in_features, int64_t rank, int w_dtype, int a_dtype, int b_dtype,
                                double scale, void* norm_out, float* parts, void* workspace, size_t workspace_bytes,
                                void* stream) {
  if (out_features < 0 || in_features < 0 || rank < 0) return DORA_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(w_dtype) || !dtype_ok(a_dtype) || !dtype_ok(b_dtype)) return DORA_ERR_INVALID_ARGUMENT;
  if (out_features == 0) return DORA_OK;
  if (!norm_out || (in_features > 0 && !W)) return DORA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t M = out_features, K = in_features, R = rank;
  int rc0;
  const bool lora_term = scale != 0.0 && R > 0 && K > 0;
  if (lora_term && (!A || !B)) return DORA_ERR_INVALID_ARGUMENT;
  NormPlan p = make_plan(M, K, R, w_dtype, a_dtype, b_dtype, true);
  const bool aligned = aligned16(W) && (!lora_term || ((p.cast_a || aligned16(A)) && (p.cast_b || aligned16(B))));
  if (!aligned) p = make_plan(M, K, R, w_dtype, a_dtype, b_dtype, false);
  if (!workspace || workspace_bytes < p.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return DORA_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  if (lora_term && p.cast_a) {
    // 0. fp32 adapters rounded into the weight dtype (workspace copies, 16-byte aligned).
    launch_cast_to_half(static_cast<const float*>(A), ws + p.off_a, R * K, w_dtype, st);
    if ((rc0 = check_launch())) return rc0;
    A = ws + p.off_a;
    a_dtype = w_dtype;
  }
  if (lora_term && p.cast_b) {
    launch_cast_to_half(static_cast<const float*>(B), ws + p.off_bh, M * R, w_dtype, st);
    if ((rc0 = check_launch())) return rc0;
    B = ws + p.off_bh;
    b_dtype = w_dtype;
  }
  float* gpart = reinterpret_cast<float*>(ws + p.off_gpart);
  float* yt = reinterpret_cast<float*>(ws + p.off_yt);
  void* hi = ws + p.off_hi;
  void* lo = ws + p.off_lo;
  float* wpart = reinterpret_cast<float*>(ws + p.off_w);
  float* cpart = reinterpret_cast<float*>(ws + p.off_c);
  float* bpart = reinterpret_cast<float*>(ws + p.off_b);
  int rc;

  if (!lora_term) {
    // ||W0|| only: the scale == 0 short-cut (dora.py:1117-1129), or no adapter rank.
    if (K > 0) {
      launch_row_sumsq(w_dtype, W, M, K, wpart, st);
      if ((rc = check_launch())) return rc;
    }
    launch_norm_finalize(wpart, K > 0 ? 1 : 0, cpart, 0, bpart, 0, M, scale, w_dtype, norm_out, parts, st);
    return check_launch();
  }

  if (p.fuse_g) {
    // Low rank: cross term, ||W0||^2 and partial Grams in one stream-K launch, then the
    // finalize with B G B^T.
    float* g16 = reinterpret_cast<float*>(ws + p.off_g16);
    TcGemmArgs u{};
    u.dtype = w_dtype; u.X = W; u.Y1 = A; u.Y2 = nullptr; u.Z = B; u.ldz = R;
    u.M = M; u.N = R; u.K = K; u.mode = kGemmRowdot; u.sumsq = true; u.k_splits = p.u_splits;
    u.rowdot_part = cpart; u.sumsq_part = wpart; u.g_part = g16;
    if (!tc_sk_supported(u)) return DORA_ERR_INVALID_ARGUMENT;
    if ((rc = tc_sk_rowdot_gemm(u, p.sk, st))) return rc;
    launch_norm_finalize_gram(wpart, p.u_splits, cpart, p.u_splits * p.u_ntiles, g16, p.sk.grid, int(R), B, b_dtype,
                              M, scale, w_dtype, norm_out, parts, st);
    return check_launch();
  }

  // 1-2. Gram matrix G = A A^T.
  if (p.tc_g) {
    TcGemmArgs g{};
    g.dtype = a_dtype; g.X = A; g.Y1 = A; g.Y2 = nullptr; g.Z = nullptr; g.ldz = 0;
    g.M = R; g.N = R; g.K = K; g.mode = kGemmStore; g.sumsq = false; g.k_splits = p.gram_splits;
    g.C = gpart; g.tri = true;
    if ((rc = tc_rowdot_gemm(g, st))) return rc;
  } else {
    simt_gemm<kGemmStore, false>(a_dtype, a_dtype, a_dtype, A, K, A, K, nullptr, 0, R, R, K, p.gram_splits,
                                 nullptr, nullptr, gpart, R, st);
    if ((rc = check_launch())) return rc;
  }
  launch_gram_reduce(gpart, p.gram_splits, R, yt, p.tc_v ? b_dtype : DORA_DTYPE_BF16, p.tc_v ? hi : nullptr,
                     p.tc_v ? lo : nullptr, p.tc_g ? kGramTile : 0, st);
  if ((rc = check_launch())) return rc;

  // 3. cross term + ||W0||^2.
  if (p.tc_u) {
    TcGemmArgs u{};
    u.dtype = w_dtype; u.X = W; u.Y1 = A; u.Y2 = nullptr; u.Z = B; u.ldz = R;
    u.M = M; u.N = R; u.K = K; u.mode = kGemmRowdot; u.sumsq = true; u.k_splits = p.u_splits;
    u.rowdot_part = cpart; u.sumsq_part = wpart;
    if (p.fuse_v) {
      u.G1 = hi; u.G2 = lo; u.v_part = bpart;
    }
    if (p.pair_u && tc2_supported(u)) rc = tc2_rowdot_gemm(u, st);
    else if (p.pair_u) return DORA_ERR_INVALID_ARGUMENT;  // planned for pairs, but B is misaligned
    else if (p.sk2_u && tc2_sk_supported(u)) rc = tc2_sk_rowdot_gemm(u, p.sk, st);
    else if (p.sk2_u) return DORA_ERR_INVALID_ARGUMENT;
    else if (p.sk_u && tc_sk_supported(u)) rc = tc_sk_rowdot_gemm(u, p.sk, st);
    else if (p.sk_u) return DORA_ERR_INVALID_ARGUMENT;
    else rc = tc_rowdot_gemm(u, st);
    if (rc) return rc;
  } else {
    simt_gemm<kGemmRowdot, true>(w_dtype, a_dtype, b_dtype, W, K, A, K, B, R, M, R, K, p.u_splits, cpart, wpart,
                                 nullptr, 0, st);
    if ((rc = check_launch())) return rc;
  }

  // 4. B G B^T term (already done above when fused).
  if (p.fuse_v) {
  } else if (p.v_pair) {
    // An ordinary launch: it reads G's halves from the Gram reduce, which the stream-K
    // cross-term kernel before it does not wait for, so it waits for everything before
    // it; the finalize after it then sees every partial.
    TcGemmArgs v{};
    v.dtype = b_dtype; v.X = B; v.Y1 = hi; v.Y2 = lo; v.Z = B; v.ldz = R;
    v.M = M; v.N = R; v.K = R; v.mode = kGemmRowdot; v.sumsq = true; v.k_splits = p.v_splits;
    v.rowdot_part = bpart;
    v.sumsq_part = reinterpret_cast<float*>(ws + p.off_vs);
    v.plain_launch = true;
    if (!tc2_sk_supported(v)) return DORA_ERR_INVALID_ARGUMENT;
    if ((rc = tc2_sk_rowdot_gemm(v, p.vsk, st))) return rc;
  } else if (p.tc_v) {
    TcGemmArgs v{};
    v.dtype = b_dtype; v.X = B; v.Y1 = hi; v.Y2 = lo; v.Z = B; v.ldz = R;
    v.M = M; v.N = R; v.K = R; v.mode = kGemmRowdot; v.sumsq = false; v.k_splits = p.v_splits;
    v.rowdot_part = bpart;
    if ((rc = tc_rowdot_gemm(v, st))) return rc;
  } else {
    simt_gemm<kGemmRowdot, false>(b_dtype, DORA_DTYPE_F32, b_dtype, B, R, yt, R, B, R, M, R, R, 1, bpart, nullptr,
                                  nullptr, 0, st);
    if ((rc = check_launch())) return rc;
  }

  // 5. Fixed-order reduction of the partials and the norm assembly.
  launch_norm_finalize(wpart, p.u_splits, cpart, p.u_splits * p.u_ntiles, bpart, p.v_splits * p.v_ntiles, M, scale,
                       w_dtype, norm_out, parts, st);
  return check_launch();
}
