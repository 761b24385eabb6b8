// Stream-K form of the tensor-core row-dot kernel for the factored norm's cross
// term (with the fused B G B^T phase and ||W0||^2).
//
// The work of one 128-row tile is a row of "units": its kb_total k-blocks of
// X Y^T (W0 A^T) followed, when the B G B^T phase is fused, by its 2 x
// ceil(N / 64) k-blocks of Z G^T (B times the hi and lo halves of G).  Both kinds
// cost one 128 x NT x 64 MMA block.  The units of all tiles, tile after tile, are
// cut into `grid` equal contiguous ranges, one per CTA (one CTA per SM), so every
// SM gets the same amount of MMA work whatever the tile count, and a CTA pays
// its prologue (barrier set-up, TMEM allocation, pipeline fill) once.
//
// A CTA's range crosses at most a few tile boundaries; the part of the range
// inside one tile is a "segment".  Per segment:
//   mainloop   TMA ring of X / Y stages, tcgen05.mma into TMEM (fp32), row
//              warps sum the squares of the staged X rows (||W0||^2);
//   staging    once the ring is idle, the tile's Z rows (B) come into it through
//              TMA, then the G k-blocks of the segment double-buffered behind it;
//   epilogue   rowsum(acc * Z) for the segment's X Y^T units, then the segment's
//              Z G^T units accumulate in the same TMEM columns and are contracted
//              the same way.
// Segment s of a tile (s = 0 for the CTA that starts the tile) writes partial
// slot s of each row; the slots a tile does not use are zero-filled by its
// slot-0 segment, so the finalize kernel sums a fixed number of slots in a fixed
// order (the result is deterministic for a given grid size).
//
// Every mbarrier wait is bounded (about a second); on expiry the kernel records
// DORA_ERR_DEVICE_TIMEOUT, stops issuing work, drains what it issued and
// returns.  No cluster, no multicast.
#include <atomic>
#include <type_traits>

#include "tc_common.cuh"

namespace dora {
namespace tc {

// Units [sk_begin(c), sk_begin(c + 1)) belong to CTA c.
__host__ __device__ inline int64_t sk_begin(int64_t c, int64_t total, int64_t grid) { return c * total / grid; }
// The CTA whose range holds unit x.
__host__ __device__ inline int64_t sk_owner(int64_t x, int64_t total, int64_t grid) {
  int64_t c = x * grid / total;
  while (c + 1 < grid && sk_begin(c + 1, total, grid) <= x) ++c;
  while (c > 0 && sk_begin(c, total, grid) > x) --c;
  return c;
}

struct SkArgs {
  int64_t M, N;
  int nt, ybox, m_tiles, n_tiles, kblocks, stages, grid, slots;
  int ksub;            // 64-deep k-blocks per unit (one ring stage); kblocks counts units
  int apart;           // Z and the G slots have their own region after the ring (else they reuse the ring)
  uint32_t stage_off;  // Z / G region, from the 1024-aligned base
  uint32_t bar_off;    // barriers, from the 1024-aligned base
  int fuse_v, v_kblocks;
  int64_t units_per_tile, total_units;
  uint32_t tmem_cols;
  float* rowdot_part;  // [slots * n_tiles][M], entry (slot * n_tiles + n_tile)
  float* sumsq_part;   // [slots][M] (from the n_tile = 0 tiles)
  float* v_part;       // [slots][M] when fuse_v
  // Low-rank Gram (nt == 16, no fused B G B^T): every CTA writes its partial
  // G = sum A_k A_k^T over the k-blocks it is responsible for, [grid][16 x 16].
  int fuse_g, kb_total;
  float* g_part;
  // With fuse_g the row threads read their B row (nt = 16 values) from here into
  // registers at each segment start instead of staging the B tile: the ring never
  // drains between segments.
  const void* zsrc;
};

// The tile whose CTA adds k-block kb of A to its partial Gram: k-blocks are spread
// evenly over the tiles, so every CTA gets about the same share.
__host__ __device__ inline int64_t gram_tile(int64_t kb, int64_t kb_total, int64_t m_tiles) {
  return kb * m_tiles / kb_total;
}

__host__ __device__ inline uint32_t sk_stage_bytes(int nt) { return kXTileBytes + uint32_t(nt) * 128u; }

// Shared-memory layout: a ring of `stages` X / Y stages, then (when the tile is
// narrow enough) a separate region for the staged Z rows and two G slots, so
// the next segment's ring loads can stream in while this segment's epilogue
// runs; wide tiles stage Z / G in the idle ring instead.
// At most 12 stages; narrow tiles fill the ring with fewer, deeper stages instead
// (sk_layout below).
constexpr int kMaxSkStages = 12;

struct SkLayout {
  int stages, apart, ksub;
  uint32_t stage_off, bar_off, total;
};
inline SkLayout sk_layout_k(int nt, bool fuse_v, int ksub) {
  const uint32_t budget = 220u * 1024u;
  const uint32_t stage = sk_stage_bytes(nt) * uint32_t(ksub);
  const uint32_t z_bytes = uint32_t((nt + BK - 1) / BK) * kXTileBytes;
  const uint32_t staging = z_bytes + (fuse_v ? 2u * uint32_t(nt) * 128u : 0u);
  SkLayout L{};
  int s_apart = staging < budget ? int((budget - staging) / stage) : 0;
  if (s_apart > kMaxSkStages) s_apart = kMaxSkStages;
  if (s_apart >= 4) {
    L.stages = s_apart;
    L.apart = 1;
    L.stage_off = stage * uint32_t(s_apart);
    L.bar_off = L.stage_off + staging;
  } else {
    int s = int(budget / stage);
    L.stages = s > kMaxSkStages ? kMaxSkStages : s;
    L.apart = 0;
    L.stage_off = 0;
    L.bar_off = stage * uint32_t(L.stages);
  }
  L.total = 1024u + L.bar_off + 512u;  // barriers (2 per stage + 10) and two words
  L.ksub = ksub;
  return L;
}

// Units (ring stages) of up to four 64-deep k-blocks, as many as keep three stages in
// flight.  Every unit pays a fixed hand-off (TMA issue, MMA issue and commit, the row
// sums' release), which narrow tiles do not hide behind their few bytes per k-block:
// at 28672 x 8192 bf16, r = 16 went from 0.169 to 0.140 ms with four k-blocks per unit,
// r = 128 from 0.183 to 0.161 ms with two.  Below 256 columns two k-blocks per unit pay
// even with only two stages (r = 192: 0.202 -> 0.184 ms); wider tiles keep one.
inline SkLayout sk_layout(int nt, bool fuse_v) {
  for (int k = 4; k > 1; --k) {
    const SkLayout L = sk_layout_k(nt, fuse_v, k);
    if (L.stages >= 3) return L;
  }
  if (nt < 256) {
    const SkLayout L = sk_layout_k(nt, fuse_v, 2);
    if (L.stages >= 2) return L;
  }
  return sk_layout_k(nt, fuse_v, 1);
}

template <typename T, bool kSumSq>
__global__ void __launch_bounds__(kThreads, 1)
tc_sk_rowdot_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmY,
                    const __grid_constant__ CUtensorMap tmZ, const __grid_constant__ CUtensorMap tmG1,
                    const __grid_constant__ CUtensorMap tmG2, const SkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nt = a.nt, S = a.stages;
  const uint32_t sub_bytes = sk_stage_bytes(nt);  // one 64-deep k-block of X and Y
  const int ksub = a.ksub;
  const uint32_t stage_bytes = sub_bytes * uint32_t(ksub);
  uint8_t* zbase = base + a.stage_off;  // staged Z rows, then two G slots
  uint64_t* full = reinterpret_cast<uint64_t*>(base + a.bar_off);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;       // MMA -> rows: the segment's X Y^T units are accumulated
  uint64_t* zfull = done + 1;       // producer -> all: the segment's Z rows are staged
  uint64_t* vfull = zfull + 1;      // [2] G k-block slots
  uint64_t* vempty = vfull + 2;     // [2]
  uint64_t* tmem_free = vempty + 2; // rows -> MMA: first epilogue done with TMEM
  uint64_t* vdone = tmem_free + 1;  // MMA -> rows: the segment's Z G^T units are accumulated
  uint64_t* seg_free = vdone + 1;   // rows -> producer, MMA: TMEM and staged Z no longer read
  uint64_t* drain = seg_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* aborted = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = blockIdx.x;
  const int64_t TU = a.units_per_tile, TOT = a.total_units, G = a.grid;
  const int kbt = a.kblocks;  // X Y^T units per tile; the rest of a tile's units are Z G^T
  const int vkb = a.v_kblocks;
  const int nzb = (nt + BK - 1) / BK;
  const uint32_t z_bytes = uint32_t(nzb) * kXTileBytes;
  const uint32_t vslot_bytes = uint32_t(nt) * 128u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + (kSumSq ? 4 : 0));
    }
    mbar_init(done, 1);
    mbar_init(zfull, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    mbar_init(tmem_free, 4);
    mbar_init(vdone, 1);
    mbar_init(seg_free, 4);
    mbar_init(drain, 1);
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
  pdl_trigger();

  const int64_t u_first = sk_begin(c, TOT, G), u_last = sk_begin(c + 1, TOT, G);
  // Segment `seg` of this CTA: tile, tile-local unit range [ua, ub), its X Y^T
  // part [ua, min(ub, kbt)) and its Z G^T part [max(ua, kbt), ub) - kbt.
  struct Seg {
    int64_t tile, m_tile;
    int n_tile, ua, ub, u_iters, v0, v_iters;
  };
  // Tiles run N-tile fastest, so the N tiles of one row block stream the same W0
  // rows close together in time (L2 reuse).
  auto segment = [&](int64_t u) {
    Seg s;
    s.tile = u / TU;
    s.m_tile = s.tile / a.n_tiles;
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
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmY)) : "memory");
      int64_t gk = 0, gv = 0;  // ring uses and G slot uses so far
      int z_seg = -1;  // segment whose Z staging load this thread issued last
      int seg = 0;
      for (int64_t u = u_first; u < u_last && !*aborted; ++seg) {
        const Seg sg = segment(u);
        u = sg.tile * TU + sg.ub;
        const int m0 = int(sg.m_tile * BM);
        const int n0 = sg.n_tile * nt;
        // Ring mode: the previous segment's epilogues must be done with the staged Z / G
        // (which live in the ring) before the ring is refilled.
        if (!a.fuse_g && !a.apart && seg > 0 && !mbar_wait(seg_free, (seg - 1) & 1)) { *aborted = 1; break; }
        for (int i = 0; i < sg.u_iters; ++i) {
          const int64_t g = gk;
          const int s = int(g % S);
          if (g >= S && !mbar_wait(&empty[s], uint32_t((g / S - 1) & 1))) { *aborted = 1; break; }
          if (*aborted) break;
          uint8_t* stage = base + size_t(s) * stage_bytes;
          // The last unit's k-blocks past K read the fill value (zero) and count in full.
          mbar_expect_tx(&full[s], stage_bytes);
          for (int h = 0; h < ksub; ++h) {
            const int kx = ((sg.ua + i) * ksub + h) * BK;
            uint8_t* sX = stage + size_t(h) * sub_bytes;
            tma_load_2d(sX, &tmX, &full[s], kx, m0);
            for (int j = 0; j * a.ybox < nt; ++j)
              tma_load_2d(sX + kXTileBytes + size_t(j) * a.ybox * 128, &tmY, &full[s], kx, n0 + j * a.ybox);
          }
          ++gk;
          // Start the tile's Z rows towards L2 a few k-blocks before they are staged.
          if (i == (sg.u_iters > S + 1 ? sg.u_iters - S - 1 : 0))
            for (int j = 0; j < nzb; ++j) tma_prefetch_2d(&tmZ, n0 + j * BK, m0);
        }
        if (*aborted) break;
        if (a.fuse_g) continue;  // no B tile to stage: the next segment's loads follow at once
        bool ok = true;
        if (a.apart) {
          // Own region: only the previous segment's epilogues have to be done with it.
          if (seg > 0) ok = mbar_wait(seg_free, (seg - 1) & 1);
        } else {
          // Ring idle: every issued X / Y stage has been consumed by the MMAs (and the row sums).
          for (int64_t g = gk - S > 0 ? gk - S : 0; g < gk && ok; ++g)
            ok = mbar_wait(&empty[g % S], uint32_t((g / S) & 1));
        }
        if (!ok) { *aborted = 1; break; }
        mbar_expect_tx(zfull, z_bytes);
        for (int j = 0; j < nzb; ++j) tma_load_2d(zbase + size_t(j) * kXTileBytes, &tmZ, zfull, n0 + j * BK, m0);
        z_seg = seg;
        for (int i = 0; i < sg.v_iters; ++i) {
          if (gv == 0) pdl_wait();  // G (hi / lo) is written by the previous kernel
          const int64_t g = gv;
          const int vs = int(g & 1);
          if (g >= 2 && !mbar_wait(&vempty[vs], uint32_t((g / 2 - 1) & 1))) { *aborted = 1; break; }
          const int kv = sg.v0 + i;
          const bool lo = kv >= vkb;
          const int kx = (lo ? kv - vkb : kv) * BK;
          uint8_t* slot = zbase + z_bytes + size_t(vs) * vslot_bytes;
          mbar_expect_tx(&vfull[vs], vslot_bytes);
          const CUtensorMap* gm = lo ? &tmG2 : &tmG1;
          for (int j = 0; j * a.ybox < nt; ++j)
            tma_load_2d(slot + size_t(j) * a.ybox * 128, gm, &vfull[vs], kx, j * a.ybox);
          ++gv;
        }
      }
      // Let every copy this thread issued land before the CTA's shared memory goes away.
      for (int64_t g = gk - S > 0 ? gk - S : 0; g < gk; ++g) mbar_wait(&full[g % S], uint32_t((g / S) & 1));
      if (z_seg >= 0) mbar_wait(zfull, uint32_t(z_seg & 1));
      for (int64_t g = gv - 2 > 0 ? gv - 2 : 0; g < gv; ++g) mbar_wait(&vfull[g & 1], uint32_t((g / 2) & 1));
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool bf16 = std::is_same<T, __nv_bfloat16>::value;
      const MmaChunks chunks = mma_chunks(bf16, nt, BM);
      int64_t gk = 0, gv = 0;
      int n_tf = 0;  // tmem_free phases consumed
      int seg = 0;
      bool ok = true;
      for (int64_t u = u_first; u < u_last && ok; ++seg) {
        const Seg sg = segment(u);
        u = sg.tile * TU + sg.ub;
        if (seg > 0 && !mbar_wait(seg_free, (seg - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        for (int i = 0; i < sg.u_iters; ++i) {
          const int64_t g = gk++;
          const int s = int(g % S);
          if (!mbar_wait(&full[s], uint32_t((g / S) & 1))) { ok = false; break; }
          tc_fence_after();
          const uint32_t stage = smem_u32(base + size_t(s) * stage_bytes);
          for (int h = 0; h < ksub; ++h) {
            const uint32_t sX = stage + uint32_t(h) * sub_bytes;
            mma_kblock(tmem_base, sX, sX + kXTileBytes, chunks, i > 0 || h > 0);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        if (sg.u_iters > 0) umma_commit(done);
        if (sg.v_iters > 0) {
          if (!mbar_wait(zfull, seg & 1)) { ok = false; break; }
          if (sg.u_iters > 0) {
            if (!mbar_wait(tmem_free, n_tf & 1)) { ok = false; break; }
            ++n_tf;
          }
          tc_fence_after();
          for (int i = 0; i < sg.v_iters; ++i) {
            const int64_t g = gv++;
            const int vs = int(g & 1);
            if (!mbar_wait(&vfull[vs], uint32_t((g / 2) & 1))) { ok = false; break; }
            tc_fence_after();
            const int kv = sg.v0 + i;
            const int kz = kv >= vkb ? kv - vkb : kv;  // k-block of Z (= column block of B)
            const uint32_t sA = smem_u32(zbase + size_t(kz) * kXTileBytes);
            const uint32_t sB = smem_u32(zbase + z_bytes + size_t(vs) * vslot_bytes);
            mma_kblock(tmem_base, sA, sB, chunks, i > 0);
            umma_commit(&vempty[vs]);
          }
          if (!ok) break;
          umma_commit(vdone);
        }
      }
      if (!ok) *aborted = 1;
      umma_commit(drain);  // completes once every MMA issued above has finished
      mbar_wait(drain, 0);
    }
  } else {
    // ------------------------------------------------------------ row threads
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16);
    int cur_n0 = 0;  // first column of the current segment's N tile
    auto rowdot_epilogue = [&]() -> float {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int64_t ncols = a.N - cur_n0;
      int c0 = 0;
      for (; c0 + 64 <= int(a.tmem_cols) && c0 < nt && c0 < ncols; c0 += 64) {
        float v[64];
        tmem_ld64(trow + uint32_t(c0), v);
        const int cnt = (ncols - c0) < 64 ? int(ncols - c0) : 64;
        dot_staged<T, 64>(v, zbase, c0, row, cnt, acc);
      }
      for (; c0 < nt && c0 < ncols; c0 += 32) {
        float v[32];
        tmem_ld32(trow + uint32_t(c0), v);
        const int cnt = (ncols - c0) < 32 ? int(ncols - c0) : 32;
        dot_staged<T, 32>(v, zbase, c0, row, cnt, acc);
      }
      return sum8(acc);
    };
    int64_t gk = 0;
    int n_done = 0, n_vdone = 0;
    int seg = 0;
    // Partial Gram entries of this thread: G[ga][gb] and G[ga][gb + 1] (nt == 16:
    // 128 row threads x 2 = all 256 entries).
    const int ga = row >> 3, gb = (row & 7) * 2;
    float g0 = 0.f, g1 = 0.f;
    for (int64_t u = u_first; u < u_last; ++seg) {
      const Seg sg = segment(u);
      u = sg.tile * TU + sg.ub;
      const int64_t m = sg.m_tile * BM + row;
      cur_n0 = sg.n_tile * nt;
      // fuse_g: this row's N (8 or 16) B values; rows are N * 2 bytes, 16-byte aligned.
      uint4 zr0 = make_uint4(0u, 0u, 0u, 0u), zr1 = zr0;
      if (a.fuse_g && m < a.M) {
        const uint4* zp = reinterpret_cast<const uint4*>(static_cast<const T*>(a.zsrc) + m * a.N);
        zr0 = __ldg(zp);
        if (a.N > 8) zr1 = __ldg(zp + 1);
      }
      const bool ssq_tile = sg.n_tile == 0;  // ||X||^2 once per row block
      // k-blocks [kg_lo, kg_hi) of A go into this tile's partial Gram (gram_tile(kb) == m_tile).
      int kg_lo = 0, kg_hi = 0;
      if (a.fuse_g) {
        kg_lo = int((sg.m_tile * a.kb_total + a.m_tiles - 1) / a.m_tiles);
        kg_hi = int(((sg.m_tile + 1) * a.kb_total + a.m_tiles - 1) / a.m_tiles);
      }
      float ssq8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight independent FMA chains
      bool ok = true;
      if (kSumSq) {
        for (int i = 0; i < sg.u_iters; ++i) {
          const int64_t g = gk++;
          const int s = int(g % S);
          // Every ring use is released by the row warps too (fixed barrier count); the
          // data is summed only in the N tile that owns ||X||^2.
          if (!warp_wait(&full[s], uint32_t((g / S) & 1))) { ok = false; break; }
          if (!ssq_tile) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            continue;
          }
          for (int hb = 0; hb < ksub; ++hb) {
            const uint8_t* rowp = base + size_t(s) * stage_bytes + size_t(hb) * sub_bytes + row * 128;
#pragma unroll
            for (int p = 0; p < 8; ++p) {
              // Rotate the 16-byte chunk order by lane so a quarter-warp touches 8 distinct bank groups.
              const uint4 v = *reinterpret_cast<const uint4*>(rowp + ((p + lane) & 7) * 16);
              sumsq8<T>(v, ssq8);
            }
            {
              // This k-block's A rows are staged right after its X tile (16 rows of
              // 128 bytes, 128-byte swizzle: chunk c of row q at c ^ (q & 7)).
              const int kb = (sg.ua + i) * ksub + hb;
              if (kb >= kg_lo && kb < kg_hi) {
                const uint8_t* ay = base + size_t(s) * stage_bytes + size_t(hb) * sub_bytes + kXTileBytes;
#pragma unroll
                for (int p = 0; p < 8; ++p) {
                  const uint4 va = *reinterpret_cast<const uint4*>(ay + ga * 128 + ((p ^ (ga & 7)) * 16));
                  const uint4 vb0 = *reinterpret_cast<const uint4*>(ay + gb * 128 + ((p ^ (gb & 7)) * 16));
                  const uint4 vb1 =
                      *reinterpret_cast<const uint4*>(ay + (gb + 1) * 128 + ((p ^ ((gb + 1) & 7)) * 16));
                  const T* xa = reinterpret_cast<const T*>(&va);
                  const T* x0 = reinterpret_cast<const T*>(&vb0);
                  const T* x1 = reinterpret_cast<const T*>(&vb1);
#pragma unroll
                  for (int e = 0; e < 8; ++e) {
                    const float av = to_f32(xa[e]);
                    g0 = fmaf(av, to_f32(x0[e]), g0);
                    g1 = fmaf(av, to_f32(x1[e]), g1);
                  }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
      }
      const int64_t first = sk_owner(sg.tile * TU, TOT, G);
      const int slot = int(c - first);
      ok = ok && __all_sync(0xffffffffu, !*aborted && (a.fuse_g || mbar_wait(zfull, seg & 1)) &&
                                             (sg.u_iters == 0 || mbar_wait(done, n_done & 1)));
      if (!ok) {
        *aborted = 1;
        break;
      }
      if (sg.u_iters > 0) ++n_done;
      tc_fence_after();
      float cacc = 0.f;
      if (a.fuse_g) {
        // 16 accumulator columns; TMEM goes back to the MMA warp as soon as it is read,
        // so the next segment's MMAs overlap this dot (same order as dot_staged).
        float v[32];
        tmem_ld32(trow, v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(seg_free);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const T* z0 = reinterpret_cast<const T*>(&zr0);
        const T* z1 = reinterpret_cast<const T*>(&zr1);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(v[e], to_f32(z0[e]), acc[e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(v[8 + e], to_f32(z1[e]), acc[e]);
        cacc = sum8(acc);
      } else if (sg.u_iters > 0) {
        cacc = rowdot_epilogue();
      }
      if (m < a.M) {
        a.rowdot_part[(int64_t(slot) * a.n_tiles + sg.n_tile) * a.M + m] = cacc;
        if (ssq_tile) a.sumsq_part[int64_t(slot) * a.M + m] = sum8(ssq8);
      }
      float bacc = 0.f;
      if (sg.v_iters > 0) {
        if (sg.u_iters > 0) {
          // Hand the TMEM columns to the Z G^T units.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tmem_free);
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
        // Zero the slots this tile does not use, so the finalize sums a fixed count.
        const int used = int(sk_owner(sg.tile * TU + TU - 1, TOT, G) - first) + 1;
        for (int s2 = used; s2 < a.slots; ++s2) {
          a.rowdot_part[(int64_t(s2) * a.n_tiles + sg.n_tile) * a.M + m] = 0.f;
          if (ssq_tile) a.sumsq_part[int64_t(s2) * a.M + m] = 0.f;
          if (a.fuse_v) a.v_part[int64_t(s2) * a.M + m] = 0.f;
        }
      }
      if (!a.fuse_g) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(seg_free);
      }
    }
    if (a.fuse_g) {
      // Every CTA writes its slot (zeros when it had no Gram k-blocks), so the
      // finalize sums a fixed number of partials in a fixed order.
      a.g_part[c * 256 + ga * 16 + gb] = g0;
      a.g_part[c * 256 + ga * 16 + gb + 1] = g1;
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


}  // namespace tc

bool tc_sk_supported(const TcGemmArgs& a) {
  if (a.mode != kGemmRowdot || !a.sumsq || a.Y2 || !a.Z || a.ldz != a.N || (a.ldz * 2) % 16 != 0 ||
      !aligned16(a.Z))
    return false;
  const TcGemmShape sh = tc_gemm_shape(a.M, a.N, a.K);
  if (sh.n_tiles != 1 && a.G1) return false;  // the fused B G B^T phase needs the whole row in one tile
  const tc::SkLayout L = tc::sk_layout(sh.nt, a.G1 != nullptr);
  const uint32_t z_bytes = uint32_t((sh.nt + tc::BK - 1) / tc::BK) * tc::kXTileBytes;
  const uint32_t staging = z_bytes + (a.G1 ? 2u * uint32_t(sh.nt) * 128u : 0u);
  if (L.stages < 2 || (!L.apart && staging > L.bar_off)) return false;
  if (a.G1 && (!a.G2 || !a.v_part || !tc_can_fuse_v(a.M, a.N, a.K))) return false;
  return true;
}

SkPlan tc_sk_plan(int64_t M, int64_t N, int64_t K, bool fuse_v, int sms) {
  const TcGemmShape sh = tc_gemm_shape(M, N, K);
  SkPlan p;
  const int ksub = tc::sk_layout(sh.nt, fuse_v).ksub;
  p.units_per_tile = int64_t((sh.kblocks + ksub - 1) / ksub) + (fuse_v ? 2 * ((N + tc::BK - 1) / tc::BK) : 0);
  const int64_t tiles = int64_t(sh.m_tiles) * sh.n_tiles;
  p.total_units = tiles * p.units_per_tile;
  // One CTA per SM, but no CTA with fewer than four units (each segment pays a staging and epilogue).
  int64_t g = p.total_units / 4;
  if (g > sms) g = sms;
  if (g < 1) g = 1;
  p.grid = int(g);
  int slots = 1;
  for (int64_t t = 0; t < tiles; ++t) {
    const int64_t f = tc::sk_owner(t * p.units_per_tile, p.total_units, g);
    const int64_t l = tc::sk_owner(t * p.units_per_tile + p.units_per_tile - 1, p.total_units, g);
    if (int(l - f + 1) > slots) slots = int(l - f + 1);
  }
  p.slots = slots;
  return p;
}

template <typename T, bool SSQ>
static int launch_sk(const tc::SkArgs& k, const CUtensorMap* m, cudaStream_t st, bool pdl) {
  const uint32_t smem = 1024u + k.bar_off + 512u;
  auto kfn = tc::tc_sk_rowdot_kernel<T, SSQ>;
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
  // Launched as a programmatic dependent of the Gram reduce: the X Y^T units start at
  // once, the producer waits for the reduce only before its first G load.  With the
  // Gram fused in (low rank) it is the chain's first kernel: an ordinary launch, which
  // waits for whatever wrote W0, A and B before it.
  if (pdl)
    e = launch_pdl(kfn, dim3(unsigned(k.grid)), dim3(tc::kThreads), smem, st, m[0], m[1], m[2], m[3], m[4], k);
  else {
    kfn<<<dim3(unsigned(k.grid)), dim3(tc::kThreads), smem, st>>>(m[0], m[1], m[2], m[3], m[4], k);
    e = cudaSuccess;
  }
  if (e != cudaSuccess) return set_cuda_error(e);
  return check_launch();
}

int tc_sk_rowdot_gemm(const TcGemmArgs& a, const SkPlan& p, cudaStream_t st) {
  if (!tc_sk_supported(a)) return DORA_ERR_UNSUPPORTED;
  const TcGemmShape sh = tc_gemm_shape(a.M, a.N, a.K);
  const int ybox = sh.nt <= 256 ? sh.nt : 128;
  const bool fuse = a.G1 != nullptr;
  CUtensorMap maps[5];
  if (!tc::make_map(&maps[0], a.X, a.dtype, a.M, a.K, tc::BM) || !tc::make_map(&maps[1], a.Y1, a.dtype, a.N, a.K, ybox) ||
      !tc::make_map(&maps[2], a.Z, a.dtype, a.M, a.ldz, tc::BM))
    return DORA_ERR_CUDA;
  maps[3] = maps[1];
  maps[4] = maps[1];
  if (fuse && (!tc::make_map(&maps[3], a.G1, a.dtype, a.N, a.N, ybox) ||
               !tc::make_map(&maps[4], a.G2, a.dtype, a.N, a.N, ybox)))
    return DORA_ERR_CUDA;
  tc::SkArgs k{};
  k.M = a.M;
  k.N = a.N;
  k.nt = sh.nt;
  k.ybox = ybox;
  k.m_tiles = sh.m_tiles;
  k.n_tiles = sh.n_tiles;
  const tc::SkLayout L = tc::sk_layout(sh.nt, fuse);
  k.ksub = L.ksub;
  k.kblocks = (sh.kblocks + L.ksub - 1) / L.ksub;  // units of ksub k-blocks
  k.stages = L.stages;
  k.apart = L.apart;
  k.stage_off = L.stage_off;
  k.bar_off = L.bar_off;
  k.grid = p.grid;
  k.slots = p.slots;
  k.fuse_v = fuse ? 1 : 0;
  k.v_kblocks = int((a.N + tc::BK - 1) / tc::BK);
  k.units_per_tile = int64_t(k.kblocks) + (fuse ? 2 * k.v_kblocks : 0);
  k.total_units = int64_t(sh.m_tiles) * sh.n_tiles * k.units_per_tile;
  if (k.units_per_tile != p.units_per_tile || k.total_units != p.total_units) return DORA_ERR_INVALID_ARGUMENT;
  uint32_t cols = 32;
  while (cols < uint32_t(sh.nt)) cols <<= 1;
  k.tmem_cols = cols;
  k.rowdot_part = a.rowdot_part;
  k.sumsq_part = a.sumsq_part;
  k.v_part = a.v_part;
  k.fuse_g = a.g_part ? 1 : 0;
  k.kb_total = sh.kblocks;
  k.g_part = a.g_part;
  k.zsrc = a.Z;
  if (k.fuse_g && (fuse || sh.nt != 16 || ybox != 16)) return DORA_ERR_INVALID_ARGUMENT;
  if (a.dtype == DORA_DTYPE_BF16) return launch_sk<__nv_bfloat16, true>(k, maps, st, !k.fuse_g);
  return launch_sk<__half, true>(k, maps, st, !k.fuse_g);
}

}  // namespace dora
