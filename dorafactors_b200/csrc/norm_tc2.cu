// CTA-pair (cta_group::2) row-dot GEMM for the factored DoRA norm.
//
// Same computation as the single-CTA kernel in norm_tc.cu (C = X Y^T contracted
// row by row with Z, ||X||^2 fused, optional B G B^T phase), but two CTAs of a
// cluster share each MMA: the pair covers 256 rows, each CTA stages its own 128
// rows of X and HALF of the Y tile, and the leader CTA (rank 0) issues
// tcgen05.mma.cta_group::2 with M = 256.  Per k-block a CTA therefore loads
// 16 KB + nt/2 x 128 B instead of 16 KB + nt x 128 B (40 KB instead of 64 KB at
// r = 384), which lets the ring hold five stages instead of three: the
// single-CTA kernel is limited by load latency, not bandwidth.
//
// Synchronisation (all waits bounded):
//   full[s]    leader only; the leader expects both CTAs' bytes, every load of
//              either CTA counts on it (cta_group::2 TMA, no multicast);
//   mdone[s]   both CTAs; the leader's commit arrives on both when the MMAs that
//              read slot s finish;
//   empty[s]   both CTAs; the row-sum warps release slot s after reading X;
//   done/vdone both CTAs; commits after the last MMA of each phase;
//   zfull      local; this CTA's staged Z tile;
//   peer_z     leader; the peer reports its Z tile has landed;
//   vfull/vempty the B G B^T phase's G slots, same pattern as full/mdone;
//   tmem_free  leader; all 8 epilogue warps have drained the first product;
//   teardown   each CTA waits for the other before the paired TMEM free.
#include <atomic>
#include <type_traits>

#include "tc_common.cuh"

namespace dora {
namespace tc {

struct PairLayout {
  uint32_t stage_bytes;
  uint32_t ring_bytes;
  uint32_t total;
};
__host__ __device__ inline PairLayout pair_layout(int nt, int stages) {
  PairLayout L;
  L.stage_bytes = kXTileBytes + uint32_t(nt) * 64u;  // X tile + half of the Y tile
  L.ring_bytes = L.stage_bytes * uint32_t(stages);
  L.total = 1024u + L.ring_bytes + 512u;
  return L;
}
inline int pair_stages(int nt) {
  int s = int((220u * 1024u) / pair_layout(nt, 1).stage_bytes);
  return s > 8 ? 8 : s;
}

struct PArgs {
  const void* Z;
  int64_t ldz;
  int64_t M, N;
  int nt, hb, n_tiles, m_pairs, kblocks, k_splits, stages;
  int two_y, z_tma, fuse_v, v_kblocks;
  uint32_t tmem_cols;
  float* rowdot_part;
  float* sumsq_part;
  float* v_part;
};

template <typename T, bool kSumSq>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
tc2_rowdot_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY1,
                  const __grid_constant__ CUtensorMap tmY2, const __grid_constant__ CUtensorMap tmZ,
                  const __grid_constant__ CUtensorMap tmG1, const __grid_constant__ CUtensorMap tmG2,
                  const PArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nt = a.nt, stages = a.stages;
  const PairLayout L = pair_layout(nt, stages);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.ring_bytes);
  uint64_t* mdone = full + stages;
  uint64_t* empty = mdone + stages;
  uint64_t* done = empty + stages;
  uint64_t* drain = done + 1;
  uint64_t* zfull = drain + 1;
  uint64_t* peer_z = zfull + 1;
  uint64_t* vfull = peer_z + 1;   // [2]
  uint64_t* vempty = vfull + 2;   // [2]
  uint64_t* tmem_free = vempty + 2;
  uint64_t* vdone = tmem_free + 1;
  uint64_t* teardown = vdone + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(teardown + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int unit = blockIdx.x >> 1;
  const int m_pair = unit % a.m_pairs;
  const int rest = unit / a.m_pairs;
  const int n_tile = rest % a.n_tiles;
  const int ks = rest / a.n_tiles;
  const int64_t m0 = int64_t(m_pair) * 2 * BM + int64_t(rank) * BM;  // this CTA's rows
  const int64_t n0 = int64_t(n_tile) * nt;
  const int kb_total = a.two_y ? 2 * a.kblocks : a.kblocks;
  const int kb0 = int(int64_t(ks) * kb_total / a.k_splits);
  const int iters = int(int64_t(ks + 1) * kb_total / a.k_splits) - kb0;
  const bool do_ssq = kSumSq && n_tile == 0;
  const int vk_total = a.fuse_v ? 2 * a.v_kblocks : 0;
  const int vk0 = int(int64_t(ks) * vk_total / a.k_splits);
  const int v_iters = int(int64_t(ks + 1) * vk_total / a.k_splits) - vk0;
  const uint32_t z_bytes = uint32_t((nt + BK - 1) / BK) * kXTileBytes;
  const uint32_t vhalf = uint32_t(nt) * 64u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&mdone[s], 1);
      mbar_init(&empty[s], 4);
    }
    mbar_init(done, 1);
    mbar_init(drain, 1);
    mbar_init(zfull, 1);
    mbar_init(peer_z, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    mbar_init(tmem_free, 8);
    mbar_init(vdone, 1);
    mbar_init(teardown, 1);
    *aborted = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Y (and G) halves: CTA r stages rows [r * nt/2, (r + 1) * nt/2) of the tile as
  // one box.  Its first N0/2 rows (N0 = min(nt, 256)) are its half of MMA chunk 0,
  // the rest its half of chunk 1, so accumulator column c holds tile row
  // pair_col_row(c, nt) -- a permutation of 64-column blocks that the epilogue
  // undoes when it picks the matching Z columns.
  auto load_half = [&](uint8_t* dst, const CUtensorMap* map, uint32_t bar_c, int kx, int row_base) {
    tma_load_2d_pair(dst, map, bar_c, kx, row_base + int(rank) * (nt / 2));
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmY1)) : "memory");
      uint64_t* release = do_ssq ? empty : mdone;  // a slot is free once this completes
      int issued = 0;
      for (int it = 0; it < iters; ++it) {
        const int s = it % stages, round = it / stages;
        if (round > 0 && !mbar_wait(&release[s], (round - 1) & 1)) { *aborted = 1; break; }
        if (*aborted) break;
        const int kb = kb0 + it;
        const bool second = kb >= a.kblocks;
        const int kx = (second ? kb - a.kblocks : kb) * BK;
        uint8_t* sX = base + size_t(s) * L.stage_bytes;
        const uint32_t bar_c = map_to_rank(&full[s], 0);
        if (leader) mbar_expect_tx(&full[s], 2u * L.stage_bytes);
        tma_load_2d_pair(sX, &tmX, bar_c, kx, int(m0));
        load_half(sX + kXTileBytes, second ? &tmY2 : &tmY1, bar_c, kx, int(n0));
        issued = it + 1;
        if (a.z_tma && it == (iters > stages + 1 ? iters - stages - 1 : 0))
          for (int j = 0; j * BK < nt; ++j) tma_prefetch_2d(&tmZ, int(n0) + j * BK, int(m0));
      }
      bool ok = !*aborted;
      if (!ok) {
        // Wait (bounded) until the MMAs that read what this CTA loaded are done.
        for (int it = issued - stages > 0 ? issued - stages : 0; it < issued; ++it)
          mbar_wait(&mdone[it % stages], (it / stages) & 1);
      } else if (a.z_tma) {
        for (int it = iters - stages > 0 ? iters - stages : 0; it < iters && ok; ++it)
          ok = mbar_wait(&release[it % stages], (it / stages) & 1);
        if (!ok) {
          *aborted = 1;
        } else {
          const int nzb = (nt + BK - 1) / BK;
          mbar_expect_tx(zfull, uint32_t(nzb) * kXTileBytes);
          for (int j = 0; j < nzb; ++j)
            tma_load_2d(base + size_t(j) * kXTileBytes, &tmZ, zfull, int(n0) + j * BK, int(m0));
          // Report the staged Z tile before loading G: the leader's MMAs need it before
          // they can release the G slots this loop waits on.
          if (!mbar_wait(zfull, 0)) {
            *aborted = 1;
          } else if (!leader) {
            mbar_arrive_remote(map_to_rank(peer_z, 0));
          }
          int v_issued = 0;
          for (int i = 0; i < v_iters; ++i) {
            const int vs = i & 1, round = i >> 1;
            if (*aborted || (round > 0 && !mbar_wait(&vempty[vs], (round - 1) & 1))) { *aborted = 1; break; }
            const int kv = vk0 + i;
            const bool lo = kv >= a.v_kblocks;
            const int kx = (lo ? kv - a.v_kblocks : kv) * BK;
            const uint32_t bar_c = map_to_rank(&vfull[vs], 0);
            if (leader) mbar_expect_tx(&vfull[vs], 2u * vhalf);
            load_half(base + z_bytes + size_t(vs) * vhalf, lo ? &tmG2 : &tmG1, bar_c, kx, 0);
            v_issued = i + 1;
          }
          // Keep this thread until its G loads have been consumed.
          for (int i = v_issued - 2 > 0 ? v_issued - 2 : 0; i < v_issued; ++i)
            mbar_wait(&vempty[i & 1], (i >> 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
      const MmaChunks chunks = mma_chunks(bf16, nt, 256);
      for (int it = 0; it < iters; ++it) {
        const int s = it % stages, round = it / stages;
        if (!mbar_wait(&full[s], round & 1)) { *aborted = 1; break; }
        tc_fence_after();
        const uint32_t sX = smem_u32(base + size_t(s) * L.stage_bytes);
        mma2_kblock(tmem_base, sX, sX + kXTileBytes, chunks, it > 0);
        umma2_commit_both(&mdone[s]);
      }
      bool ok = !*aborted;
      if (ok) umma2_commit_both(done);
      if (ok && v_iters > 0) {
        ok = mbar_wait(zfull, 0) && mbar_wait_cluster(peer_z, 0) && mbar_wait_cluster(tmem_free, 0);
        if (ok) tc_fence_after();
        for (int i = 0; ok && i < v_iters; ++i) {
          const int vs = i & 1, round = i >> 1;
          if (!mbar_wait(&vfull[vs], round & 1)) { ok = false; break; }
          tc_fence_after();
          const int kv = vk0 + i;
          const int kz = kv >= a.v_kblocks ? kv - a.v_kblocks : kv;
          const uint32_t sA = smem_u32(base + size_t(kz) * kXTileBytes);
          const uint32_t sB = smem_u32(base + z_bytes + size_t(vs) * vhalf);
          mma2_kblock(tmem_base, sA, sB, chunks, i > 0);
          umma2_commit_both(&vempty[vs]);
        }
        if (ok) umma2_commit_both(vdone);
        else *aborted = 1;
      }
      if (*aborted) {
        umma2_commit_both(drain);
        mbar_wait(drain, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ row threads (both CTAs)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int64_t m = m0 + row;
    float ssq8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight independent FMA chains
    if (do_ssq) {
      for (int it = 0; it < iters; ++it) {
        const int s = it % stages, round = it / stages;
        // The MMAs that read slot s are done, so its X tile has landed and stays until we release it.
        if (!warp_wait(&mdone[s], round & 1)) { *aborted = 1; break; }
        const uint8_t* rowp = base + size_t(s) * L.stage_bytes + row * 128;
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((p + lane) & 7) * 16);
          sumsq8<T>(v, ssq8);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
    const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16);
    auto rowdot_epilogue = [&]() -> float {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int64_t ncols = a.N - n0;
      int c0 = 0;
      for (; c0 + 64 <= int(a.tmem_cols) && c0 < nt; c0 += 64) {
        const int zc = pair_col_row(c0, nt);  // 64-column blocks map to contiguous Z columns
        if (zc >= ncols) continue;            // warp-uniform: the TMEM load is skipped by all lanes
        float v[64];
        tmem_ld64(trow + uint32_t(c0), v);
        const int cnt = (ncols - zc) < 64 ? int(ncols - zc) : 64;
        if (m < a.M) dot_staged<T, 64>(v, base, zc, row, cnt, acc);
      }
      for (; c0 < nt; c0 += 32) {  // allocations of 32 columns (nt <= 32: identity order)
        const int zc = pair_col_row(c0, nt);
        if (zc >= ncols) continue;
        float v[32];
        tmem_ld32(trow + uint32_t(c0), v);
        const int cnt = (ncols - zc) < 32 ? int(ncols - zc) : 32;
        if (m < a.M) dot_staged<T, 32>(v, base, zc, row, cnt, acc);
      }
      return sum8(acc);
    };
    const bool ok = __all_sync(0xffffffffu, !*aborted && mbar_wait(done, 0) && mbar_wait(zfull, 0));
    if (ok) {
      tc_fence_after();
      const float acc = rowdot_epilogue();
      if (m < a.M) {
        a.rowdot_part[(int64_t(ks) * a.n_tiles + n_tile) * a.M + m] = acc;
        if (do_ssq) a.sumsq_part[int64_t(ks) * a.M + m] = sum8(ssq8);
      }
      if (v_iters > 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(map_to_rank(tmem_free, 0));
        if (__all_sync(0xffffffffu, !*aborted && mbar_wait(vdone, 0))) {
          tc_fence_after();
          const float bacc = rowdot_epilogue();
          if (m < a.M) a.v_part[int64_t(ks) * a.M + m] = bacc;
        }
      } else if (a.fuse_v && m < a.M) {
        a.v_part[int64_t(ks) * a.M + m] = 0.f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) {
      // Neither CTA frees the paired TMEM (or exits) before the other is done with it.
      mbar_arrive_remote(map_to_rank(teardown, rank ^ 1u));
      mbar_wait_cluster(teardown, 0);
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(a.tmem_cols)
                 : "memory");
  }
}

}  // namespace tc

bool tc2_supported(const TcGemmArgs& a) {
  if (a.mode != kGemmRowdot || !a.Z || a.ldz != a.N || (a.ldz * 2) % 16 != 0 || !aligned16(a.Z)) return false;
  const TcGemmShape sh = tc_gemm_shape(a.M, a.N, a.K);
  if (sh.nt > 512 || a.M < 2 * tc::BM) return false;
  const int stages = tc::pair_stages(sh.nt);
  const tc::PairLayout L = tc::pair_layout(sh.nt, stages);
  const uint32_t z_bytes = uint32_t((sh.nt + tc::BK - 1) / tc::BK) * tc::kXTileBytes;
  if (stages < 2 || z_bytes > L.ring_bytes) return false;
  if (a.G1 && (sh.n_tiles != 1 || z_bytes + 2u * uint32_t(sh.nt) * 64u > L.ring_bytes || a.N % 8 != 0)) return false;
  return true;
}

int tc2_pairs(int64_t M) { return int((M + 2 * tc::BM - 1) / (2 * tc::BM)); }

template <typename T, bool SSQ>
static int launch_tc2(const tc::PArgs& k, unsigned grid, const CUtensorMap* m, cudaStream_t st) {
  const tc::PairLayout L = tc::pair_layout(k.nt, k.stages);
  auto kfn = tc::tc2_rowdot_kernel<T, SSQ>;
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
  kfn<<<grid, tc::kThreads, L.total, st>>>(m[0], m[1], m[2], m[3], m[4], m[5], k);
  return check_launch();
}

int tc2_rowdot_gemm(const TcGemmArgs& a, cudaStream_t st) {
  if (!tc2_supported(a)) return DORA_ERR_UNSUPPORTED;
  const TcGemmShape sh = tc_gemm_shape(a.M, a.N, a.K);
  const int kb_total = a.Y2 ? 2 * sh.kblocks : sh.kblocks;
  if (a.k_splits < 1 || a.k_splits > kb_total) return DORA_ERR_INVALID_ARGUMENT;
  const int hb = sh.nt / 2;  // one box per CTA half (nt <= 512, so at most 256 rows)
  CUtensorMap maps[6];
  if (!tc::make_map(&maps[0], a.X, a.dtype, a.M, a.K, tc::BM) || !tc::make_map(&maps[1], a.Y1, a.dtype, a.N, a.K, hb) ||
      !tc::make_map(&maps[2], a.Y2 ? a.Y2 : a.Y1, a.dtype, a.N, a.K, hb) ||
      !tc::make_map(&maps[3], a.Z, a.dtype, a.M, a.ldz, tc::BM))
    return DORA_ERR_CUDA;
  maps[4] = maps[0];
  maps[5] = maps[0];
  const bool fuse = a.G1 != nullptr;
  if (fuse && (!tc::make_map(&maps[4], a.G1, a.dtype, a.N, a.N, hb) ||
               !tc::make_map(&maps[5], a.G2, a.dtype, a.N, a.N, hb)))
    return DORA_ERR_CUDA;
  tc::PArgs k{};
  k.Z = a.Z;
  k.ldz = a.ldz;
  k.M = a.M;
  k.N = a.N;
  k.nt = sh.nt;
  k.hb = hb;
  k.n_tiles = sh.n_tiles;
  k.m_pairs = tc2_pairs(a.M);
  k.kblocks = sh.kblocks;
  k.k_splits = a.k_splits;
  k.stages = tc::pair_stages(sh.nt);
  k.two_y = a.Y2 ? 1 : 0;
  k.z_tma = 1;
  k.fuse_v = fuse ? 1 : 0;
  k.v_kblocks = int((a.N + tc::BK - 1) / tc::BK);
  uint32_t cols = 32;
  while (cols < uint32_t(sh.nt)) cols <<= 1;
  k.tmem_cols = cols;
  k.rowdot_part = a.rowdot_part;
  k.sumsq_part = a.sumsq_part;
  k.v_part = a.v_part;
  const unsigned grid = 2u * unsigned(k.m_pairs) * unsigned(sh.n_tiles) * unsigned(a.k_splits);
  if (a.dtype == DORA_DTYPE_BF16)
    return a.sumsq ? launch_tc2<__nv_bfloat16, true>(k, grid, maps, st) : launch_tc2<__nv_bfloat16, false>(k, grid, maps, st);
  return a.sumsq ? launch_tc2<__half, true>(k, grid, maps, st) : launch_tc2<__half, false>(k, grid, maps, st);
}

}  // namespace dora
