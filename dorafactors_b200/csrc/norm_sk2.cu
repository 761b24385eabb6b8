// Stream-K row-dot kernel on CTA pairs (cta_group::2) for the factored norm's
// cross term, ||W0||^2 and the fused B G B^T phase.
//
// The stream-K schedule of norm_sk.cu (equal contiguous shares of all tiles'
// units, segments, fixed-order partial slots) over 256-row pair tiles: a cluster
// of two CTAs on two SMs shares each MMA (M = 256, issued by rank 0), each CTA
// staging its own 128 rows of W0 and one contiguous half of A's rows, so an SM
// pulls 16 KB of W0 + nt*64 bytes of A per k-block instead of 16 KB + nt*128.
// Accumulator column c holds tile row pair_col_row(c, nt) (see tc_common.cuh);
// the epilogue reads the matching Z columns.
//
// The row sums of squares read each staged W0 tile once the MMA is done with the
// stage (`mdone`, committed to both CTAs), then release the slot (`empty`).
// Per-k-block waits use CTA-scope acquire; only the per-segment hand-offs between
// the two CTAs (Z staged, TMEM free) use cluster scope.
//
// Every wait is bounded (about a second); on expiry the kernel records
// DORA_ERR_DEVICE_TIMEOUT, stops issuing and returns.  No TMA multicast: every
// TMA load reads this GPU's global memory into the issuing CTA's own shared
// memory (the cta_group::2 form only signals the leader's barrier).
#include <atomic>
#include <cstdlib>
#include <type_traits>

#include "tc_common.cuh"

namespace dora {
namespace tc {

// Same partition helpers as the single-CTA stream-K kernel (units of pair tiles).
__host__ __device__ inline int64_t sk2_begin(int64_t c, int64_t total, int64_t grid) { return c * total / grid; }
__host__ __device__ inline int64_t sk2_owner(int64_t x, int64_t total, int64_t grid) {
  int64_t c = x * grid / total;
  while (c + 1 < grid && sk2_begin(c + 1, total, grid) <= x) ++c;
  while (c > 0 && sk2_begin(c, total, grid) > x) --c;
  return c;
}

struct Sk2Args {
  int64_t M, N;
  int nt, pair_tiles, kblocks, stages, clusters, slots;
  int n_tiles;  // N tiles of nt columns (r > 512; then no fused B G B^T phase)
  // With a second Y (Y2 in the tmG2 slot, no fused phase): the first y2_units units of a
  // tile multiply X by Y1, the next y2_units X (re-read) by Y2, into one accumulator.
  int y2_units;
  int ksub;  // 64-deep k-blocks per unit (one ring stage); kblocks counts units
  int apart;
  uint32_t stage_off, bar_off;
  int fuse_v, v_kblocks;
  int64_t units_per_tile, total_units;
  uint32_t tmem_cols;
  float* rowdot_part;  // [slots * n_tiles][M], entry (slot * n_tiles + n_tile)
  float* sumsq_part;   // [slots][M] (from the n_tile = 0 tiles)
  float* v_part;       // [slots][M] when fuse_v
};

__host__ __device__ inline uint32_t sk2_stage_bytes(int nt) { return kXTileBytes + uint32_t(nt) * 64u; }
// G k-block slots of the fused B G B^T phase (a ring of its own, staged after Z).
constexpr int kVSlots = 4;

struct Sk2Layout {
  int stages, apart, ksub;
  uint32_t stage_off, bar_off, total;
};
inline Sk2Layout sk2_layout_k(int nt, bool fuse_v, int ksub) {
  const uint32_t budget = 220u * 1024u;
  const uint32_t stage = sk2_stage_bytes(nt) * uint32_t(ksub);
  const uint32_t z_bytes = uint32_t((nt + BK - 1) / BK) * kXTileBytes;
  const uint32_t staging = z_bytes + (fuse_v ? uint32_t(kVSlots) * uint32_t(nt) * 64u : 0u);
  Sk2Layout L{};
  int s_apart = staging < budget ? int((budget - staging) / stage) : 0;
  if (s_apart > 8) s_apart = 8;
  if (s_apart >= 4) {
    L.stages = s_apart;
    L.apart = 1;
    L.stage_off = stage * uint32_t(s_apart);
    L.bar_off = L.stage_off + staging;
  } else {
    int s = int(budget / stage);
    L.stages = s > 8 ? 8 : s;
    L.apart = 0;
    L.stage_off = 0;
    L.bar_off = stage * uint32_t(L.stages);
  }
  L.total = 1024u + L.bar_off + 512u;
  L.ksub = ksub;
  return L;
}
// As in the single-CTA kernel: units of up to four k-blocks while three stages fit.
inline Sk2Layout sk2_layout(int nt, bool fuse_v) {
  for (int k = 4; k > 1; --k) {
    const Sk2Layout L = sk2_layout_k(nt, fuse_v, k);
    if (L.stages >= 3) return L;
  }
  return sk2_layout_k(nt, fuse_v, 1);
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
tc2_sk_rowdot_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY,
                     const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmG1,
                     const __grid_constant__ CUtensorMap tmG2, const Sk2Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nt = a.nt, S = a.stages;
  const uint32_t sub_bytes = sk2_stage_bytes(nt);  // one 64-deep k-block of X and this CTA's Y half
  const int ksub = a.ksub;
  const uint32_t stage_bytes = sub_bytes * uint32_t(ksub);
  uint8_t* zbase = base + a.stage_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + a.bar_off);  // leader: both halves of a stage landed
  uint64_t* mdone = full + S;       // both: the MMA finished reading the stage
  uint64_t* empty = mdone + S;      // local: the row sums finished reading the stage (after mdone)
  uint64_t* done = empty + S;       // both: the segment's X Y^T units are accumulated
  uint64_t* zfull = done + 1;       // local: this CTA's Z rows are staged
  uint64_t* peer_z = zfull + 1;     // leader: the peer's Z rows are staged
  uint64_t* vfull = peer_z + 1;            // [kVSlots] leader: both halves of a G k-block landed
  uint64_t* vempty = vfull + kVSlots;      // [kVSlots] both: the MMA finished reading a G slot
  uint64_t* tmem_free = vempty + kVSlots;  // leader: all rows of the pair finished the first epilogue
  uint64_t* vdone = tmem_free + 1;  // both: the segment's Z G^T units are accumulated
  uint64_t* seg_free = vdone + 1;   // local: this CTA's rows are done with staged Z / G
  uint64_t* tm_free = seg_free + 1; // leader: all rows of the pair are done with TMEM
  uint64_t* drain = tm_free + 1;
  uint64_t* teardown = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(teardown + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t cl = blockIdx.x >> 1;
  const int64_t TU = a.units_per_tile, TOT = a.total_units, G = a.clusters;
  const int kbt = a.kblocks, vkb = a.v_kblocks;
  const int nzb = (nt + BK - 1) / BK;
  const uint32_t z_bytes = uint32_t(nzb) * kXTileBytes;
  const uint32_t vhalf = uint32_t(nt) * 64u;
  const int half_rows = nt / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&mdone[s], 1);
      mbar_init(&empty[s], 4);
    }
    mbar_init(done, 1);
    mbar_init(zfull, 1);
    mbar_init(peer_z, 1);
    for (int s = 0; s < kVSlots; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    mbar_init(tmem_free, 8);
    mbar_init(vdone, 1);
    mbar_init(seg_free, 4);
    mbar_init(tm_free, 8);
    mbar_init(drain, 1);
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
  pdl_trigger();

  const int64_t u_first = sk2_begin(cl, TOT, G), u_last = sk2_begin(cl + 1, TOT, G);
  struct Seg {
    int64_t tile, m_pair;
    int n_tile, ua, ub, u_iters, v0, v_iters;
  };
  // Tiles run N-tile fastest: the N tiles of one pair of row blocks stream the same W0
  // rows close together in time, so only the first reads them from DRAM.
  auto segment = [&](int64_t u) {
    Seg s;
    s.tile = u / TU;
    s.m_pair = s.tile / a.n_tiles;
    s.n_tile = int(s.tile % a.n_tiles);
    s.ua = int(u - s.tile * TU);
    const int64_t e = u_last - s.tile * TU;
    s.ub = int(e < TU ? e : TU);
    const int xe = s.ub < kbt ? s.ub : kbt;
    s.u_iters = xe > s.ua ? xe - s.ua : 0;
    s.v0 = (s.ua > kbt ? s.ua : kbt) - kbt;
    s.v_iters = s.ub - kbt - s.v0 > 0 ? s.ub - kbt - s.v0 : 0;
    return s;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producers (both CTAs)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmY)) : "memory");
      int64_t gk = 0, gv = 0;
      int seg = 0;
      // A slot may be refilled once the row sums (which wait for the MMA) have released its last use.
      auto slot_free = [&](int64_t g) { return mbar_wait(&empty[g % S], uint32_t((g / S) & 1)); };
      for (int64_t u = u_first; u < u_last && !*aborted; ++seg) {
        const Seg sg = segment(u);
        u = sg.tile * TU + sg.ub;
        const int m0 = int(sg.m_pair * 2 * BM + int64_t(rank) * BM);  // this CTA's rows
        const int n0 = sg.n_tile * nt;  // first column of the N tile (row of A / Z column)
        if (!a.apart && seg > 0 && !mbar_wait(seg_free, (seg - 1) & 1)) { *aborted = 1; break; }
        for (int i = 0; i < sg.u_iters; ++i) {
          const int64_t g = gk;
          const int s = int(g % S);
          if (g >= S && !slot_free(g - S)) { *aborted = 1; break; }
          if (*aborted) break;
          uint8_t* stage = base + size_t(s) * stage_bytes;
          const uint32_t bar_c = map_to_rank(&full[s], 0);
          if (leader) mbar_expect_tx(&full[s], 2u * stage_bytes);
          const int iu = sg.ua + i;
          const bool second = a.y2_units > 0 && iu >= a.y2_units;
          const int lu = second ? iu - a.y2_units : iu;
          for (int h = 0; h < ksub; ++h) {  // k-blocks past K read zeros and count in full
            const int kx = (lu * ksub + h) * BK;
            uint8_t* sX = stage + size_t(h) * sub_bytes;
            tma_load_2d_pair(sX, &tmX, bar_c, kx, m0);
            tma_load_2d_pair(sX + kXTileBytes, second ? &tmG2 : &tmY, bar_c, kx, n0 + int(rank) * half_rows);
          }
          ++gk;
          if (i == (sg.u_iters > S + 1 ? sg.u_iters - S - 1 : 0))
            for (int j = 0; j < nzb; ++j) tma_prefetch_2d(&tmZ, n0 + j * BK, m0);
        }
        if (*aborted) break;
        bool ok = true;
        if (a.apart) {
          if (seg > 0) ok = mbar_wait(seg_free, (seg - 1) & 1);
        } else {
          for (int64_t g = gk - S > 0 ? gk - S : 0; g < gk && ok; ++g) ok = slot_free(g);
        }
        if (!ok) { *aborted = 1; break; }
        mbar_expect_tx(zfull, z_bytes);
        for (int j = 0; j < nzb; ++j) tma_load_2d(zbase + size_t(j) * kXTileBytes, &tmZ, zfull, n0 + j * BK, m0);
        // Report the staged Z rows to the leader before loading G: the leader's Z G^T
        // MMAs need both CTAs' rows before they can release the G slots waited on below.
        if (!mbar_wait(zfull, seg & 1)) { *aborted = 1; break; }
        if (!leader) mbar_arrive_remote(map_to_rank(peer_z, 0));
        for (int i = 0; i < sg.v_iters; ++i) {
          if (gv == 0) pdl_wait();  // G (hi / lo) is written by the previous kernel
          const int64_t g = gv;
          const int vs = int(g % kVSlots);
          if (g >= kVSlots && !mbar_wait(&vempty[vs], uint32_t((g / kVSlots - 1) & 1))) { *aborted = 1; break; }
          const int kv = sg.v0 + i;
          const bool lo = kv >= vkb;
          const int kx = (lo ? kv - vkb : kv) * BK;
          const uint32_t bar_c = map_to_rank(&vfull[vs], 0);
          if (leader) mbar_expect_tx(&vfull[vs], 2u * vhalf);
          tma_load_2d_pair(zbase + z_bytes + size_t(vs) * vhalf, lo ? &tmG2 : &tmG1, bar_c, kx,
                           int(rank) * half_rows);
          ++gv;
        }
      }
      // Keep this thread until the MMAs have consumed what it loaded (bounded waits).
      for (int64_t g = gk - S > 0 ? gk - S : 0; g < gk; ++g) mbar_wait(&mdone[g % S], uint32_t((g / S) & 1));
      for (int64_t g = gv - kVSlots > 0 ? gv - kVSlots : 0; g < gv; ++g)
        mbar_wait(&vempty[g % kVSlots], uint32_t((g / kVSlots) & 1));
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
      const MmaChunks chunks = mma_chunks(bf16, nt, 2 * BM);
      int64_t gk = 0, gv = 0;
      int n_tf = 0;
      int seg = 0;
      bool ok = true;
      for (int64_t u = u_first; u < u_last && ok; ++seg) {
        const Seg sg = segment(u);
        u = sg.tile * TU + sg.ub;
        if (seg > 0 && !mbar_wait_cluster(tm_free, (seg - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        for (int i = 0; i < sg.u_iters; ++i) {
          const int64_t g = gk++;
          const int s = int(g % S);
          if (!mbar_wait(&full[s], uint32_t((g / S) & 1))) { ok = false; break; }
          tc_fence_after();
          const uint32_t stage = smem_u32(base + size_t(s) * stage_bytes);
          for (int h = 0; h < ksub; ++h) {
            const uint32_t sX = stage + uint32_t(h) * sub_bytes;
            mma2_kblock(tmem_base, sX, sX + kXTileBytes, chunks, i > 0 || h > 0);
          }
          umma2_commit_both(&mdone[s]);
        }
        if (!ok) break;
        if (sg.u_iters > 0) umma2_commit_both(done);
        if (sg.v_iters > 0) {
          if (!mbar_wait(zfull, seg & 1) || !mbar_wait_cluster(peer_z, seg & 1)) { ok = false; break; }
          if (sg.u_iters > 0) {
            if (!mbar_wait_cluster(tmem_free, n_tf & 1)) { ok = false; break; }
            ++n_tf;
          }
          tc_fence_after();
          for (int i = 0; i < sg.v_iters; ++i) {
            const int64_t g = gv++;
            const int vs = int(g % kVSlots);
            if (!mbar_wait(&vfull[vs], uint32_t((g / kVSlots) & 1))) { ok = false; break; }
            tc_fence_after();
            const int kv = sg.v0 + i;
            const int kz = kv >= vkb ? kv - vkb : kv;
            const uint32_t sA = smem_u32(zbase + size_t(kz) * kXTileBytes);
            const uint32_t sB = smem_u32(zbase + z_bytes + size_t(vs) * vhalf);
            mma2_kblock(tmem_base, sA, sB, chunks, i > 0);
            umma2_commit_both(&vempty[vs]);
          }
          if (!ok) break;
          umma2_commit_both(vdone);
        }
      }
      if (!ok) *aborted = 1;
      umma2_commit_both(drain);  // completes once every MMA issued above has finished
      mbar_wait(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ row threads (both CTAs)
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16);
    const uint32_t leader_tmem_free = map_to_rank(tmem_free, 0);
    const uint32_t leader_tm_free = map_to_rank(tm_free, 0);
    int cur_n0 = 0;  // first column of the current segment's N tile
    auto rowdot_epilogue = [&]() -> float {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int64_t ncols = a.N - cur_n0;
      int c0 = 0;
      for (; c0 + 64 <= int(a.tmem_cols) && c0 < nt; c0 += 64) {
        const int zc = pair_col_row(c0, nt);
        if (zc >= ncols) continue;  // warp-uniform: the TMEM load is skipped by all lanes
        float v[64];
        tmem_ld64(trow + uint32_t(c0), v);
        const int cnt = (ncols - zc) < 64 ? int(ncols - zc) : 64;
        dot_staged<T, 64>(v, zbase, zc, row, cnt, acc);
      }
      for (; c0 < nt; c0 += 32) {
        const int zc = pair_col_row(c0, nt);
        if (zc >= ncols) continue;
        float v[32];
        tmem_ld32(trow + uint32_t(c0), v);
        const int cnt = (ncols - zc) < 32 ? int(ncols - zc) : 32;
        dot_staged<T, 32>(v, zbase, zc, row, cnt, acc);
      }
      return sum8(acc);
    };
    int64_t gk = 0;
    int n_done = 0, n_vdone = 0;
    int seg = 0;
    for (int64_t u = u_first; u < u_last; ++seg) {
      const Seg sg = segment(u);
      u = sg.tile * TU + sg.ub;
      const int64_t m = sg.m_pair * 2 * BM + int64_t(rank) * BM + row;
      cur_n0 = sg.n_tile * nt;
      const bool ssq_tile = sg.n_tile == 0;  // ||W0||^2 once per row block
      float ssq8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight independent FMA chains
      bool ok = true;
      for (int i = 0; i < sg.u_iters; ++i) {
        const int64_t g = gk++;
        const int s = int(g % S);
        if (!warp_wait(&mdone[s], uint32_t((g / S) & 1))) { ok = false; break; }
        const bool ssq_unit = ssq_tile && !(a.y2_units > 0 && sg.ua + i >= a.y2_units);  // X once
        for (int hb = 0; ssq_unit && hb < ksub; ++hb) {
          const uint8_t* rowp = base + size_t(s) * stage_bytes + size_t(hb) * sub_bytes + row * 128;
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((p + lane) & 7) * 16);
            sumsq8<T>(v, ssq8);
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      const int64_t first = sk2_owner(sg.tile * TU, TOT, G);
      const int slot = int(cl - first);
      ok = ok && __all_sync(0xffffffffu, !*aborted && mbar_wait(zfull, seg & 1) &&
                                             (sg.u_iters == 0 || mbar_wait(done, n_done & 1)));
      if (!ok) {
        *aborted = 1;
        break;
      }
      if (sg.u_iters > 0) ++n_done;
      tc_fence_after();
      const float cacc = sg.u_iters > 0 ? rowdot_epilogue() : 0.f;
      if (m < a.M) {
        a.rowdot_part[(int64_t(slot) * a.n_tiles + sg.n_tile) * a.M + m] = cacc;
        if (ssq_tile) a.sumsq_part[int64_t(slot) * a.M + m] = sum8(ssq8);
      }
      float bacc = 0.f;
      if (sg.v_iters > 0) {
        if (sg.u_iters > 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(leader_tmem_free);
        }
        if (!__all_sync(0xffffffffu, !*aborted && mbar_wait(vdone, n_vdone & 1))) {
          *aborted = 1;
          break;
        }
        ++n_vdone;
        tc_fence_after();
        bacc = rowdot_epilogue();
      }
      if (a.fuse_v && m < a.M) a.v_part[int64_t(slot) * a.M + m] = bacc;
      if (slot == 0 && m < a.M) {
        const int used = int(sk2_owner(sg.tile * TU + TU - 1, TOT, G) - first) + 1;
        for (int s2 = used; s2 < a.slots; ++s2) {
          a.rowdot_part[(int64_t(s2) * a.n_tiles + sg.n_tile) * a.M + m] = 0.f;
          if (ssq_tile) a.sumsq_part[int64_t(s2) * a.M + m] = 0.f;
          if (a.fuse_v) a.v_part[int64_t(s2) * a.M + m] = 0.f;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(seg_free);
        mbar_arrive_remote(leader_tm_free);
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

// N-tile width of the CTA-pair stream-K kernel: the whole row (up to 512 columns) by
// default, 256-column tiles above; DORA_B200_PAIR_NT=<multiple of 32, at most 256>
// splits narrower rows into tiles of that width too (then B G B^T is its own launch).
static int pair_nt_override() {
  static const int nt = [] {
    const char* e = std::getenv("DORA_B200_PAIR_NT");
    const int v = e ? std::atoi(e) : 0;
    return (v >= 32 && v <= 256 && v % 32 == 0) ? v : 0;
  }();
  return nt;
}

// DORA_B200_PAIR_WIDE=0 splits rows wider than 512 columns into 256-column N tiles
// instead of the widest equal tiles (for comparison).
static bool pair_wide_tiles() {
  static const bool on = [] {
    const char* e = std::getenv("DORA_B200_PAIR_WIDE");
    return !(e && e[0] == '0');
  }();
  return on;
}

TcGemmShape tc2_sk_shape(int64_t M, int64_t N, int64_t K) {
  const int f = pair_nt_override();
  if (f > 0 && N > f) return tc_gemm_shape(M, N, K, f);
  if (N > 512 && pair_wide_tiles()) {
    // As few N tiles as hold the row at 512 columns each, of equal width (multiples of
    // 128): fewer, wider units per k-block.
    const int64_t tiles = (N + 511) / 512;
    const int64_t w = ((N + tiles - 1) / tiles + 127) / 128 * 128;
    return tc_gemm_shape(M, N, K, int(w));
  }
  return tc_gemm_shape(M, N, K);
}

bool tc2_sk_supported(const TcGemmArgs& a) {
  if (a.mode != kGemmRowdot || !a.sumsq || !a.Z || a.ldz != a.N || (a.ldz * 2) % 16 != 0 || !aligned16(a.Z))
    return false;
  if (a.Y2 && a.G1) return false;  // a second Y shares the map slot of the fused phase's G
  const TcGemmShape sh = tc2_sk_shape(a.M, a.N, a.K);
  if (a.M < 2 * tc::BM) return false;
  if (sh.n_tiles != 1 && a.G1) return false;  // the fused B G B^T phase needs the whole row in one tile
  const tc::Sk2Layout L = tc::sk2_layout(sh.nt, a.G1 != nullptr);
  const uint32_t z_bytes = uint32_t((sh.nt + tc::BK - 1) / tc::BK) * tc::kXTileBytes;
  const uint32_t staging = z_bytes + (a.G1 ? uint32_t(tc::kVSlots) * uint32_t(sh.nt) * 64u : 0u);
  if (L.stages < 2 || (!L.apart && staging > L.bar_off)) return false;
  if (a.G1 && (!a.G2 || !a.v_part || !tc_can_fuse_v(a.M, a.N, a.K))) return false;
  return true;
}

SkPlan tc2_sk_plan(int64_t M, int64_t N, int64_t K, bool fuse_v, int sms, bool two_y) {
  const TcGemmShape sh = tc2_sk_shape(M, N, K);
  SkPlan p;
  const int64_t pair_tiles = (M + 2 * tc::BM - 1) / (2 * tc::BM);
  const int ksub = tc::sk2_layout(sh.nt, fuse_v).ksub;
  p.units_per_tile = int64_t((sh.kblocks + ksub - 1) / ksub) * (two_y ? 2 : 1) +
                     (fuse_v ? 2 * ((N + tc::BK - 1) / tc::BK) : 0);
  const int64_t tiles = pair_tiles * sh.n_tiles;
  p.total_units = tiles * p.units_per_tile;
  int64_t g = p.total_units / 4;
  if (g > sms / 2) g = sms / 2;
  if (g < 1) g = 1;
  p.grid = int(g);  // clusters of two CTAs
  int slots = 1;
  for (int64_t t = 0; t < tiles; ++t) {
    const int64_t f = tc::sk2_owner(t * p.units_per_tile, p.total_units, g);
    const int64_t l = tc::sk2_owner(t * p.units_per_tile + p.units_per_tile - 1, p.total_units, g);
    if (int(l - f + 1) > slots) slots = int(l - f + 1);
  }
  p.slots = slots;
  return p;
}

template <typename T>
static int launch_sk2(const tc::Sk2Args& k, const CUtensorMap* m, uint32_t smem, cudaStream_t st, bool plain) {
  auto kfn = tc::tc2_sk_rowdot_kernel<T>;
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
  // Programmatic dependent of the Gram reduce (see the single-CTA stream-K kernel), or an
  // ordinary launch that waits for everything before it.
  if (plain) {
    kfn<<<dim3(2u * unsigned(k.clusters)), dim3(tc::kThreads), smem, st>>>(m[0], m[1], m[2], m[3], m[4], k);
    e = cudaSuccess;
  } else {
    e = launch_pdl(kfn, dim3(2u * unsigned(k.clusters)), dim3(tc::kThreads), smem, st, m[0], m[1], m[2], m[3], m[4],
                   k);
  }
  if (e != cudaSuccess) return set_cuda_error(e);
  return check_launch();
}

int tc2_sk_rowdot_gemm(const TcGemmArgs& a, const SkPlan& p, cudaStream_t st) {
  if (!tc2_sk_supported(a)) return DORA_ERR_UNSUPPORTED;
  const TcGemmShape sh = tc2_sk_shape(a.M, a.N, a.K);
  const int hb = sh.nt / 2;  // one box of A (and G) rows per CTA half (nt <= 512)
  const bool fuse = a.G1 != nullptr;
  CUtensorMap maps[5];
  if (!tc::make_map(&maps[0], a.X, a.dtype, a.M, a.K, tc::BM) || !tc::make_map(&maps[1], a.Y1, a.dtype, a.N, a.K, hb) ||
      !tc::make_map(&maps[2], a.Z, a.dtype, a.M, a.ldz, tc::BM))
    return DORA_ERR_CUDA;
  maps[3] = maps[1];
  maps[4] = maps[1];
  if (fuse && (!tc::make_map(&maps[3], a.G1, a.dtype, a.N, a.N, hb) ||
               !tc::make_map(&maps[4], a.G2, a.dtype, a.N, a.N, hb)))
    return DORA_ERR_CUDA;
  if (a.Y2 && !tc::make_map(&maps[4], a.Y2, a.dtype, a.N, a.K, hb)) return DORA_ERR_CUDA;
  const tc::Sk2Layout L = tc::sk2_layout(sh.nt, fuse);
  tc::Sk2Args k{};
  k.M = a.M;
  k.N = a.N;
  k.nt = sh.nt;
  k.pair_tiles = int((a.M + 2 * tc::BM - 1) / (2 * tc::BM));
  k.ksub = L.ksub;
  k.kblocks = (sh.kblocks + L.ksub - 1) / L.ksub;  // units of ksub k-blocks
  k.y2_units = a.Y2 ? k.kblocks : 0;
  if (a.Y2) k.kblocks *= 2;
  k.stages = L.stages;
  k.clusters = p.grid;
  k.slots = p.slots;
  k.apart = L.apart;
  k.stage_off = L.stage_off;
  k.bar_off = L.bar_off;
  k.fuse_v = fuse ? 1 : 0;
  k.v_kblocks = int((a.N + tc::BK - 1) / tc::BK);
  k.units_per_tile = int64_t(k.kblocks) + (fuse ? 2 * k.v_kblocks : 0);
  k.n_tiles = sh.n_tiles;
  k.total_units = int64_t(k.pair_tiles) * k.n_tiles * k.units_per_tile;
  if (k.units_per_tile != p.units_per_tile || k.total_units != p.total_units) return DORA_ERR_INVALID_ARGUMENT;
  uint32_t cols = 32;
  while (cols < uint32_t(sh.nt)) cols <<= 1;
  k.tmem_cols = cols;
  k.rowdot_part = a.rowdot_part;
  k.sumsq_part = a.sumsq_part;
  k.v_part = a.v_part;
  if (a.dtype == DORA_DTYPE_BF16) return launch_sk2<__nv_bfloat16>(k, maps, L.total, st, a.plain_launch);
  return launch_sk2<__half>(k, maps, L.total, st, a.plain_launch);
}

}  // namespace dora
