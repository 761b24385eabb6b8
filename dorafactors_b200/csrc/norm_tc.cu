// Tensor-core (tcgen05 + TMEM + TMA) row-dot GEMM for the factored DoRA norm.
//
// One CTA computes a 128 x NT tile of C = X Y^T over a contiguous range of
// K, with the accumulator in tensor memory:
//   warp 0      TMA producer: 128-byte-swizzled X [128 x 64] and Y [NT x 64]
//               tiles into a multi-stage shared-memory ring (mbarrier
//               complete_tx signalling);
//   warp 1      owns the TMEM allocation and issues tcgen05.mma (kind::f16,
//               fp32 accumulate) from one thread, 4 x (NT / <=256) MMAs per
//               k-block, releasing each ring slot with tcgen05.commit;
//   warps 2..5  one thread per tile row (= TMEM lane).  While the mainloop
//               runs they add up the squares of their row of X straight from
//               the staged X tiles (||W0||^2 costs no extra HBM traffic).
//               After the last MMA they read the accumulator row with
//               tcgen05.ld and either contract it with Z (rowsum(C * Z), the
//               factored norm's cross / B G B^T terms) or store it (Gram
//               partials).
// Every mbarrier wait is bounded (about one second); on expiry the kernel
// records DORA_ERR_DEVICE_TIMEOUT in the device error word, drains what it
// issued and returns instead of hanging.  No cluster, no multicast.
#include <atomic>
#include <mutex>
#include <type_traits>

#include "tc_common.cuh"

namespace dora {
namespace tc {

struct SmemLayout {
  uint32_t stage_bytes;
  uint32_t bar_offset;  // from the 1024-aligned base
  uint32_t total;       // dynamic shared memory to request (includes alignment slack)
};
__host__ __device__ inline SmemLayout smem_layout(int nt, int stages) {
  SmemLayout L;
  L.stage_bytes = kXTileBytes + uint32_t(nt) * 128u;
  L.bar_offset = L.stage_bytes * uint32_t(stages);
  L.total = 1024u + L.bar_offset + 256u;
  return L;
}

// Scalars of one launch (the tensor maps travel as separate __grid_constant__ parameters).
struct KArgs {
  const void* Z;         // rowdot mode: [M x ldz] (B), read through tmZ when z_tma, else from global
  int64_t ldz;
  int64_t M, N;
  int nt, ybox, n_tiles, m_tiles, kblocks, k_splits, stages;
  int two_y;             // Y2 supplies k-blocks kblocks .. 2*kblocks-1
  int z_tma;             // stage Z through TMA into the idle ring for the epilogue
  int fuse_v;            // also compute rowsum(Z * (Z G^T)) with G from tmG1 (hi) + tmG2 (lo)
  int v_kblocks;         // 64-wide k-blocks of G per half (ceil(N / 64))
  uint32_t tmem_cols;
  float* rowdot_part;    // [n_tiles * k_splits][M]
  float* sumsq_part;     // [k_splits][M]
  float* v_part;         // fused B G B^T partials, [k_splits][M]
  float* C;              // store mode: [k_splits][M][N]
  int tri;               // store mode: only tiles with n_tile >= m_tile (a symmetric product)
};

template <typename T, int MODE, bool kSumSq>
__global__ void __launch_bounds__(kThreads, 1)
tc_rowdot_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY1,
                 const __grid_constant__ CUtensorMap tmY2, const __grid_constant__ CUtensorMap tmZ,
                 const __grid_constant__ CUtensorMap tmG1, const __grid_constant__ CUtensorMap tmG2,
                 const KArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nt = a.nt, stages = a.stages;
  const SmemLayout L = smem_layout(nt, stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_offset);
  uint64_t* empty = full + stages;
  uint64_t* done = empty + stages;
  uint64_t* drain = done + 1;
  uint64_t* zfull = drain + 1;
  uint64_t* vfull = zfull + 1;     // [2]
  uint64_t* vempty = vfull + 2;    // [2]
  uint64_t* tmem_free = vempty + 2;
  uint64_t* vdone = tmem_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(vdone + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x;
  int m_tile, n_tile, ks;
  if (a.tri) {
    // Upper-triangular tile pairs (i <= j) of a symmetric product, then the K split.
    const int per = a.m_tiles * (a.m_tiles + 1) / 2;
    int t = unit % per;
    ks = unit / per;
    int i = 0;
    while (t >= a.m_tiles - i) {
      t -= a.m_tiles - i;
      ++i;
    }
    m_tile = i;
    n_tile = i + t;
  } else {
    m_tile = unit % a.m_tiles;
    const int rest = unit / a.m_tiles;
    n_tile = rest % a.n_tiles;
    ks = rest / a.n_tiles;
  }
  const int64_t m0 = int64_t(m_tile) * BM;
  const int64_t n0 = int64_t(n_tile) * nt;
  const int kb_total = a.two_y ? 2 * a.kblocks : a.kblocks;
  const int kb0 = int(int64_t(ks) * kb_total / a.k_splits);
  const int iters = int(int64_t(ks + 1) * kb_total / a.k_splits) - kb0;
  const bool do_ssq = kSumSq && n_tile == 0;
  // This unit's share of the fused B G B^T k-blocks (hi half then lo half).
  const int vk_total = a.fuse_v ? 2 * a.v_kblocks : 0;
  const int vk0 = int(int64_t(ks) * vk_total / a.k_splits);
  const int v_iters = int(int64_t(ks + 1) * vk_total / a.k_splits) - vk0;
  const uint32_t z_bytes = uint32_t((nt + BK - 1) / BK) * kXTileBytes;
  const uint32_t vslot_bytes = uint32_t(nt) * 128u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + (do_ssq ? 4 : 0));
    }
    mbar_init(done, 1);
    mbar_init(drain, 1);
    mbar_init(zfull, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    mbar_init(tmem_free, 4);
    mbar_init(vdone, 1);
    *aborted = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();  // the kernel after this one (Gram reduce) may be launched

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmY1)) : "memory");
      int issued = 0;
      for (int it = 0; it < iters; ++it) {
        const int s = it % stages, round = it / stages;
        if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) { *aborted = 1; break; }
        if (*aborted) break;
        const int kb = kb0 + it;
        const bool second = kb >= a.kblocks;
        const int kx = (second ? kb - a.kblocks : kb) * BK;
        uint8_t* sX = base + size_t(s) * L.stage_bytes;
        uint8_t* sY = sX + kXTileBytes;
        mbar_expect_tx(&full[s], L.stage_bytes);
        tma_load_2d(sX, &tmX, &full[s], kx, int(m0));
        const CUtensorMap* ym = second ? &tmY2 : &tmY1;
        for (int j = 0; j * a.ybox < nt; ++j)
          tma_load_2d(sY + size_t(j) * a.ybox * 128, ym, &full[s], kx, int(n0) + j * a.ybox);
        issued = it + 1;
        // Start this tile's rows of Z on their way into L2 a few k-blocks before the
        // epilogue stages them, so the staging load after the mainloop hits L2.
        if (a.z_tma && it == (iters > stages + 1 ? iters - stages - 1 : 0))
          for (int j = 0; j * BK < nt; ++j) tma_prefetch_2d(&tmZ, int(n0) + j * BK, int(m0));
      }
      if (*aborted) {
        // Let every load this thread issued land before the CTA's shared memory is released.
        for (int it = issued - stages > 0 ? issued - stages : 0; it < issued; ++it)
          mbar_wait(&full[it % stages], (it / stages) & 1);
      } else if (a.z_tma) {
        // Stage this tile's rows of Z (= B) in the ring once the last MMAs (and
        // row-sum readers) have released every slot.
        bool free_ring = true;
        for (int it = iters - stages > 0 ? iters - stages : 0; it < iters && free_ring; ++it)
          free_ring = mbar_wait(&empty[it % stages], (it / stages) & 1);
        if (!free_ring) {
          *aborted = 1;
        } else {
          const int nzb = (nt + BK - 1) / BK;
          mbar_expect_tx(zfull, uint32_t(nzb) * kXTileBytes);
          for (int j = 0; j < nzb; ++j)
            tma_load_2d(base + size_t(j) * kXTileBytes, &tmZ, zfull, int(n0) + j * BK, int(m0));
          // G tiles for the fused B G B^T phase, double-buffered after the Z tile.
          int v_issued = 0;
          for (int i = 0; i < v_iters; ++i) {
            const int vs = i & 1, round = i >> 1;
            if (round > 0 && !mbar_wait(&vempty[vs], (round - 1) & 1)) { *aborted = 1; break; }
            const int kv = vk0 + i;
            const bool lo = kv >= a.v_kblocks;
            const int kx = (lo ? kv - a.v_kblocks : kv) * BK;
            uint8_t* slot = base + z_bytes + size_t(vs) * vslot_bytes;
            mbar_expect_tx(&vfull[vs], vslot_bytes);
            const CUtensorMap* gm = lo ? &tmG2 : &tmG1;
            for (int j = 0; j * a.ybox < nt; ++j)
              tma_load_2d(slot + size_t(j) * a.ybox * 128, gm, &vfull[vs], kx, j * a.ybox);
            v_issued = i + 1;
          }
          // Keep this thread until its copies have landed.
          mbar_wait(zfull, 0);
          for (int i = v_issued - 2 > 0 ? v_issued - 2 : 0; i < v_issued; ++i) mbar_wait(&vfull[i & 1], (i >> 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
      const MmaChunks chunks = mma_chunks(bf16, nt, BM);
      for (int it = 0; it < iters; ++it) {
        const int s = it % stages, round = it / stages;
        if (!mbar_wait(&full[s], round & 1)) { *aborted = 1; break; }
        tc_fence_after();
        const uint32_t sX = smem_u32(base + size_t(s) * L.stage_bytes);
        mma_kblock(tmem_base, sX, sX + kXTileBytes, chunks, it > 0);
        umma_commit(&empty[s]);
      }
      bool ok = !*aborted;
      if (ok) umma_commit(done);
      // Fused B G B^T: Z (resident, [128 x N] in 64-column boxes) times G tiles,
      // into the same TMEM columns once the epilogue has drained the first product.
      if (ok && v_iters > 0) {
        ok = mbar_wait(zfull, 0) && mbar_wait(tmem_free, 0);
        if (ok) tc_fence_after();
        for (int i = 0; ok && i < v_iters; ++i) {
          const int vs = i & 1, round = i >> 1;
          if (!mbar_wait(&vfull[vs], round & 1)) { ok = false; break; }
          tc_fence_after();
          const int kv = vk0 + i;
          const int kz = kv >= a.v_kblocks ? kv - a.v_kblocks : kv;  // k-block of Z (= column block of B)
          const uint32_t sA = smem_u32(base + size_t(kz) * kXTileBytes);
          const uint32_t sB = smem_u32(base + z_bytes + size_t(vs) * vslot_bytes);
          mma_kblock(tmem_base, sA, sB, chunks, i > 0);
          umma_commit(&vempty[vs]);
        }
        if (ok) umma_commit(vdone);
        else *aborted = 1;
      }
      if (*aborted) {
        umma_commit(drain);  // completes once every MMA issued above has finished
        mbar_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ row threads
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int64_t m = m0 + row;
    float ssq8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight independent FMA chains
    if (do_ssq) {
      for (int it = 0; it < iters; ++it) {
        const int s = it % stages, round = it / stages;
        if (!warp_wait(&full[s], round & 1)) { *aborted = 1; break; }
        const uint8_t* rowp = base + size_t(s) * L.stage_bytes + row * 128;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          // Rotate the 16-byte chunk order by lane so a quarter-warp touches 8 distinct bank groups.
          const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((p + lane) & 7) * 16);
          sumsq8<T>(v, ssq8);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
    const T* Zg = static_cast<const T*>(a.Z);
    const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16);
    // Row dot of the accumulator row with this row of Z: staged Z (64-column boxes,
    // 128-byte rows, 16-byte chunk c of row r stored at c ^ (r % 8)) or global Z.
    auto rowdot_epilogue = [&]() -> float {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int64_t ncols = a.N - n0;  // columns of this tile inside N
      int c0 = 0;
      // 64 columns per TMEM load while the allocation holds them, then 32.
      for (; c0 + 64 <= int(a.tmem_cols) && c0 < nt && c0 < ncols; c0 += 64) {
        float v[64];
        tmem_ld64(trow + uint32_t(c0), v);
        const int cnt = (ncols - c0) < 64 ? int(ncols - c0) : 64;
        if (m < a.M) {
          if (a.z_tma) dot_staged<T, 64>(v, base, c0, row, cnt, acc);
          else dot_global<T, 64>(v, Zg + m * a.ldz + n0 + c0, cnt, acc);
        }
      }
      for (; c0 < nt && c0 < ncols; c0 += 32) {
        float v[32];
        tmem_ld32(trow + uint32_t(c0), v);
        const int cnt = (ncols - c0) < 32 ? int(ncols - c0) : 32;
        if (m < a.M) {
          if (a.z_tma) dot_staged<T, 32>(v, base, c0, row, cnt, acc);
          else dot_global<T, 32>(v, Zg + m * a.ldz + n0 + c0, cnt, acc);
        }
      }
      return sum8(acc);
    };
    const bool ok = __all_sync(0xffffffffu, !*aborted && mbar_wait(done, 0) && (!a.z_tma || mbar_wait(zfull, 0)));
    if (ok) {
      tc_fence_after();
      if constexpr (MODE == kGemmRowdot) {
        const float acc = rowdot_epilogue();
        if (m < a.M) {
          a.rowdot_part[(int64_t(ks) * a.n_tiles + n_tile) * a.M + m] = acc;
          if (do_ssq) a.sumsq_part[int64_t(ks) * a.M + m] = sum8(ssq8);
        }
        if (v_iters > 0) {
          // Hand the TMEM columns to the fused phase, then contract its product.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tmem_free);
          if (__all_sync(0xffffffffu, !*aborted && mbar_wait(vdone, 0))) {
            tc_fence_after();
            const float bacc = rowdot_epilogue();
            if (m < a.M) a.v_part[int64_t(ks) * a.M + m] = bacc;
          }
        } else if (a.fuse_v && m < a.M) {
          a.v_part[int64_t(ks) * a.M + m] = 0.f;  // this split holds no G k-blocks
        }
      } else {
        // Store mode: stage the warp's 32 x 32 block in the idle ring and write it
        // one 128-byte row per instruction.
        float* stg = reinterpret_cast<float*>(base) + q * (32 * 33);
        for (int c0 = 0; c0 < nt; c0 += 32) {
          if (n0 + c0 >= a.N) break;
          float v[32];
          tmem_ld32(trow + uint32_t(c0), v);
#pragma unroll
          for (int j = 0; j < 32; ++j) stg[lane * 33 + j] = v[j];
          __syncwarp();
          const int64_t nbase = n0 + c0;
          const int cnt = (a.N - nbase) < 32 ? int(a.N - nbase) : 32;
          for (int rr = 0; rr < 32; ++rr) {
            const int64_t mr = m0 + q * 32 + rr;
            if (mr < a.M && lane < cnt) a.C[(int64_t(ks) * a.M + mr) * a.N + nbase + lane] = stg[rr * 33 + lane];
          }
          __syncwarp();
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(a.tmem_cols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int stages_for(int nt) {
  const uint32_t stage = kXTileBytes + uint32_t(nt) * 128u;
  int s = int((220u * 1024u) / stage);
  if (s > 8) s = 8;
  return s;
}

}  // namespace tc

TcGemmShape tc_gemm_shape(int64_t M, int64_t N, int64_t K, int force_nt) {
  TcGemmShape s;
  if (force_nt > 0 && N > force_nt) {
    s.nt = force_nt;
    s.n_tiles = int((N + force_nt - 1) / force_nt);
  } else if (N <= 256) {
    s.nt = int((N + 15) / 16 * 16);
    s.n_tiles = 1;
  } else if (N <= 512) {
    s.nt = int((N + 127) / 128 * 128);
    s.n_tiles = 1;
  } else {
    s.nt = 256;
    s.n_tiles = int((N + 255) / 256);
  }
  s.m_tiles = int((M + tc::BM - 1) / tc::BM);
  s.kblocks = int((K + tc::BK - 1) / tc::BK);
  return s;
}

bool tc_gemm_supported(int dtype, int64_t M, int64_t N, int64_t K, const void* X, const void* Y, const void* Z,
                       int64_t ldz) {
  if (dtype != DORA_DTYPE_BF16 && dtype != DORA_DTYPE_F16) return false;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (K % 8 != 0) return false;  // TMA row stride must be a multiple of 16 bytes
  if (M > (int64_t(1) << 31) - 1 || N > (int64_t(1) << 31) - 1 || K > (int64_t(1) << 31) - 1) return false;
  if (!aligned16(X) || !aligned16(Y)) return false;
  (void)Z;
  (void)ldz;
  return true;
}

template <typename T, int MODE, bool SSQ>
static int launch_tc(const tc::KArgs& k, unsigned grid, const CUtensorMap& mx, const CUtensorMap& my1,
                     const CUtensorMap& my2, const CUtensorMap& mz, const CUtensorMap& mg1, const CUtensorMap& mg2,
                     cudaStream_t st) {
  const tc::SmemLayout L = tc::smem_layout(k.nt, k.stages);
  auto kfn = tc::tc_rowdot_kernel<T, MODE, SSQ>;
  // Opt in to the largest dynamic shared memory once per device for this kernel.
  static std::atomic<unsigned long long> opted{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(opted.load(std::memory_order_relaxed) & bit)) {
    e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(tc::kMaxDynamicSmem));
    if (e != cudaSuccess) return set_cuda_error(e);
    opted.fetch_or(bit, std::memory_order_relaxed);
  }
  kfn<<<grid, tc::kThreads, L.total, st>>>(mx, my1, my2, mz, mg1, mg2, k);
  return check_launch();
}

template <typename T>
static int dispatch_tc(const TcGemmArgs& a, const tc::KArgs& k, unsigned grid, const CUtensorMap& mx,
                       const CUtensorMap& my1, const CUtensorMap& my2, const CUtensorMap& mz, const CUtensorMap& mg1,
                       const CUtensorMap& mg2, cudaStream_t st) {
  if (a.mode == kGemmStore) return launch_tc<T, kGemmStore, false>(k, grid, mx, my1, my2, mz, mg1, mg2, st);
  if (a.sumsq) return launch_tc<T, kGemmRowdot, true>(k, grid, mx, my1, my2, mz, mg1, mg2, st);
  return launch_tc<T, kGemmRowdot, false>(k, grid, mx, my1, my2, mz, mg1, mg2, st);
}

bool tc_can_fuse_v(int64_t M, int64_t N, int64_t K) {
  const TcGemmShape sh = tc_gemm_shape(M, N, K);
  if (sh.n_tiles != 1 || sh.nt > 384 || N % 8 != 0) return false;
  const int stages = tc::stages_for(sh.nt);
  const uint32_t z_bytes = uint32_t((sh.nt + tc::BK - 1) / tc::BK) * tc::kXTileBytes;
  return z_bytes + 2u * uint32_t(sh.nt) * 128u <= tc::smem_layout(sh.nt, stages).bar_offset;
}

int tc_rowdot_gemm(const TcGemmArgs& a, cudaStream_t st) {
  const TcGemmShape sh = tc_gemm_shape(a.M, a.N, a.K, a.tri ? kGramTile : 0);
  if (a.tri && (a.mode != kGemmStore || a.M != a.N || sh.m_tiles != sh.n_tiles)) return DORA_ERR_INVALID_ARGUMENT;
  const int kb_total = a.Y2 ? 2 * sh.kblocks : sh.kblocks;
  if (a.k_splits < 1 || a.k_splits > kb_total) return DORA_ERR_INVALID_ARGUMENT;
  const int ybox = sh.nt <= 256 ? sh.nt : 128;
  CUtensorMap mx, my1, my2;
  if (!tc::make_map(&mx, a.X, a.dtype, a.M, a.K, tc::BM) || !tc::make_map(&my1, a.Y1, a.dtype, a.N, a.K, ybox) ||
      !tc::make_map(&my2, a.Y2 ? a.Y2 : a.Y1, a.dtype, a.N, a.K, ybox))
    return DORA_ERR_CUDA;
  const int stages = tc::stages_for(sh.nt);
  // The epilogue's Z rows come through TMA into the freed stage ring when Z's rows
  // are 16-byte aligned (a 2-D map needs a 16-byte row stride) and the tile fits.
  CUtensorMap mz = mx, mg1 = mx, mg2 = mx;
  int z_tma = 0, fuse_v = 0;
  const uint32_t z_bytes = uint32_t((sh.nt + tc::BK - 1) / tc::BK) * tc::kXTileBytes;
  if (a.mode == kGemmRowdot && a.Z && a.ldz == a.N && (a.ldz * 2) % 16 == 0 && aligned16(a.Z) &&
      z_bytes <= tc::smem_layout(sh.nt, stages).bar_offset) {
    if (!tc::make_map(&mz, a.Z, a.dtype, a.M, a.ldz, tc::BM)) return DORA_ERR_CUDA;
    z_tma = 1;
  }
  if (z_tma && a.G1 && a.G2 && a.v_part && tc_can_fuse_v(a.M, a.N, a.K)) {
    if (!tc::make_map(&mg1, a.G1, a.dtype, a.N, a.N, ybox) || !tc::make_map(&mg2, a.G2, a.dtype, a.N, a.N, ybox))
      return DORA_ERR_CUDA;
    fuse_v = 1;
  } else if (a.G1) {
    return DORA_ERR_INVALID_ARGUMENT;  // the caller asked for the fused phase on a shape that cannot hold it
  }
  tc::KArgs k{};
  k.Z = a.Z;
  k.ldz = a.ldz;
  k.M = a.M;
  k.N = a.N;
  k.nt = sh.nt;
  k.ybox = ybox;
  k.n_tiles = sh.n_tiles;
  k.m_tiles = sh.m_tiles;
  k.kblocks = sh.kblocks;
  k.k_splits = a.k_splits;
  k.stages = stages;
  k.two_y = a.Y2 ? 1 : 0;
  k.z_tma = z_tma;
  k.fuse_v = fuse_v;
  k.v_kblocks = int((a.N + tc::BK - 1) / tc::BK);
  uint32_t cols = 32;
  while (cols < uint32_t(sh.nt)) cols <<= 1;
  k.tmem_cols = cols;
  k.rowdot_part = a.rowdot_part;
  k.sumsq_part = a.sumsq_part;
  k.v_part = a.v_part;
  k.C = a.C;
  k.tri = a.tri ? 1 : 0;
  const unsigned tiles = a.tri ? unsigned(sh.m_tiles * (sh.m_tiles + 1) / 2) : unsigned(sh.m_tiles) * unsigned(sh.n_tiles);
  const unsigned grid = tiles * unsigned(a.k_splits);
  if (a.dtype == DORA_DTYPE_BF16) return dispatch_tc<__nv_bfloat16>(a, k, grid, mx, my1, my2, mz, mg1, mg2, st);
  return dispatch_tc<__half>(a, k, grid, mx, my1, my2, mz, mg1, mg2, st);
}

}  // namespace dora
