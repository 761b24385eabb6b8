// Device helpers shared by the tcgen05 kernels: mbarriers with bounded waits,
// TMA tile loads, shared-memory matrix descriptors, UMMA issue / commit and
// TMEM loads.  Single-CTA forms and the CTA-pair (cta_group::2) forms.
#pragma once

#include <mutex>
#include <type_traits>

#include "norm_internal.cuh"

namespace dora {
namespace tc {


constexpr int BM = 128;
constexpr int BK = 64;  // 64 half-precision elements = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr uint32_t kXTileBytes = BM * BK * 2;
constexpr long long kWaitCycles = 1ll << 31;
constexpr uint32_t kMaxDynamicSmem = 227u * 1024u;  // per-block opt-in limit on sm_100

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase of the given parity to complete, for at most ~2^31 cycles.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      record_device_error(DORA_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
}

// A whole warp waits for a phase: lane 0 polls the barrier (bounded, as above) and
// the other lanes follow through the warp barrier, which orders their later shared-
// memory reads after lane 0's acquire.  One polling lane instead of 32 keeps the
// row warps' spinning off the shared-memory pipe the MMAs and TMA writes use
// (≈2 % of the stream-K kernels' time at 28672 x 8192, r = 384).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  bool ok = true;
  if ((threadIdx.x & 31u) == 0u) ok = mbar_wait(bar, parity);
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok;
}

// Row sums of squares: acc[e] += x_e * x_e for the eight half-precision values in v,
// one mixed-precision FMA (half inputs, fp32 addend and result) per element.  Half
// values are exact in fp32, so each step equals fmaf(float(x), float(x), acc[e]) bit
// for bit, without a conversion instruction per element.
template <typename T>
__device__ __forceinline__ void sumsq8(const uint4& v, float* acc) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
      asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
          "fma.rn.f32.bf16 %0, l, l, %0;\n\tfma.rn.f32.bf16 %1, h, h, %1;\n\t}"
          : "+f"(acc[2 * j]), "+f"(acc[2 * j + 1])
          : "r"(w[j]));
    else
      asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
          "fma.rn.f32.f16 %0, l, l, %0;\n\tfma.rn.f32.f16 %1, h, h, %1;\n\t}"
          : "+f"(acc[2 * j]), "+f"(acc[2 * j + 1])
          : "r"(w[j]));
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major tile stored as 128-byte rows
// in the 128-byte swizzle pattern (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B): 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);   // start address
  d |= uint64_t(1) << 16;                  // leading byte offset (unused when swizzled)
  d |= uint64_t(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                  // descriptor version for sm_100
  d |= uint64_t(2) << 61;                  // swizzle mode: 128 B
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator, A/B both bf16 or both
// f16, both K-major, M = m (128 for one CTA, 256 for a CTA pair), N = n.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, int n, int m = BM) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Load 32 (64) consecutive fp32 accumulator columns of this warp's 32 TMEM lanes
// (one row per thread).  The wait is part of the same asm statement, so the
// outputs are defined only once the load has completed.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, "
      "[%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// Prefetch one tile of a tensor map into L2 (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// Row-dot epilogue pieces: accumulate v[j] * z[j] over NC accumulator columns
// into eight independent partial sums (one per element of a 16-byte chunk),
// so the FMA dependence chain is NC / 8 long instead of NC.  Columns at or
// beyond `cnt` are skipped.
//
// Staged Z: 64-column boxes of 128-byte rows, 16-byte chunk c of row r stored
// at c ^ (r % 8) (the TMA 128-byte swizzle); c0 is a multiple of NC.
template <typename T, int NC>
__device__ __forceinline__ void dot_staged(const float (&v)[NC], const uint8_t* ztile, int c0, int row, int cnt,
                                           float (&acc)[8]) {
  const uint8_t* zrow = ztile + size_t(c0 / BK) * kXTileBytes + row * 128;
  const int q0 = (c0 % BK) / 8;
  if (cnt >= NC) {
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) {
      const uint4 zv = *reinterpret_cast<const uint4*>(zrow + (((q0 + j) ^ (row & 7)) * 16));
      const T* zh = reinterpret_cast<const T*>(&zv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(v[j * 8 + e], to_f32(zh[e]), acc[e]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) {
      const uint4 zv = *reinterpret_cast<const uint4*>(zrow + (((q0 + j) ^ (row & 7)) * 16));
      const T* zh = reinterpret_cast<const T*>(&zv);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (j * 8 + e < cnt) acc[e] = fmaf(v[j * 8 + e], to_f32(zh[e]), acc[e]);
    }
  }
}
// Z row read from global memory (zr points at column c0 of this thread's row).
template <typename T, int NC>
__device__ __forceinline__ void dot_global(const float (&v)[NC], const T* zr, int cnt, float (&acc)[8]) {
  if (cnt >= NC && (reinterpret_cast<uintptr_t>(zr) & 15u) == 0) {
#pragma unroll
    for (int j = 0; j < NC / 8; ++j) {
      const uint4 zv = __ldg(reinterpret_cast<const uint4*>(zr) + j);
      const T* zh = reinterpret_cast<const T*>(&zv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(v[j * 8 + e], to_f32(zh[e]), acc[e]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < NC; ++j)
      if (j < cnt) acc[j & 7] = fmaf(v[j], to_f32(zr[j]), acc[j & 7]);
  }
}
__device__ __forceinline__ float sum8(const float (&acc)[8]) {
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}


// ---------------------------------------------------------------------------
// CTA-pair (cta_group::2) forms.  The two CTAs of a cluster of two share one
// MMA: rank 0 (the leader) issues it, each CTA supplies half of the operands
// from its own shared memory and receives its half of the rows in its TMEM.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a local barrier that the peer CTA arrives on.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      record_device_error(DORA_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
  return true;
}
// TMA tile load into this CTA's shared memory whose completion is counted on a
// barrier of either CTA of the pair (cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once MMAs issued so far complete) on the barrier at this offset in both CTAs.
__device__ __forceinline__ void umma2_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Tile row (= column of A, G and Z) held in accumulator column c when each CTA of
// the pair stages one contiguous half of the tile's B-operand rows: chunk 0
// (N0 = min(nt, 256) columns) takes rows [0, N0/2) from CTA 0 and [nt/2, nt/2 +
// N0/2) from CTA 1; chunk 1 (nt - N0 columns) takes the next rows of each half.
// The identity for nt <= 256; a swap of 64-column-aligned blocks for nt = 384, 512.
__host__ __device__ inline int pair_col_row(int c, int nt) {
  const int n0 = nt < 256 ? nt : 256, h0 = n0 / 2, half = nt / 2;
  if (c < n0) return c < h0 ? c : half + (c - h0);
  const int i = c - n0, h1 = (nt - n0) / 2;
  return i < h1 ? h0 + i : half + h0 + (i - h1);
}

// ---------------------------------------------------------------------------
// One 64-deep k-block of MMAs into an NT-column accumulator (NT <= 512): at most
// two column chunks (N <= 256 each), instruction descriptors computed once.
// The issue loop has a fixed trip count and no per-MMA arithmetic beyond the
// descriptor start address: written as a loop bounded by NT at run time, the
// same MMAs kept the tensor pipe only ~60 % busy (1254 instead of 769 SM
// cycles per 128 x 384 x 64 k-block, measured with operands resident in shared
// memory), because the single issuing thread could not feed it back to back.
// ---------------------------------------------------------------------------
struct MmaChunks {
  uint32_t id0, id1;  // instruction descriptors of columns [0, 256) and [256, NT)
  bool two;
};
__device__ __forceinline__ MmaChunks mma_chunks(bool bf16, int nt, int m) {
  MmaChunks c;
  c.id0 = make_idesc(bf16, nt < 256 ? nt : 256, m);
  c.id1 = make_idesc(bf16, nt > 256 ? nt - 256 : 16, m);
  c.two = nt > 256;
  return c;
}
// Single CTA (M = 128): A [128 x 64] at sA, B [NT x 64] at sB, both 128-byte
// swizzled K-major tiles.
__device__ __forceinline__ void mma_kblock(uint32_t tmem, uint32_t sA, uint32_t sB, const MmaChunks& c,
                                           bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < BK / 16; ++kk) {
    const uint64_t ad = sw128_desc(sA + kk * 32);
    const uint32_t acc = (accumulate || kk > 0) ? 1u : 0u;
    umma_f16(tmem, ad, sw128_desc(sB + kk * 32), c.id0, acc);
    if (c.two) umma_f16(tmem + 256u, ad, sw128_desc(sB + 256u * 128u + kk * 32), c.id1, acc);
  }
}
// CTA pair (M = 256, issued by the leader): each CTA holds half of every
// column chunk's B rows, so chunk 1 starts 128 rows into the local B tile.
__device__ __forceinline__ void mma2_kblock(uint32_t tmem, uint32_t sA, uint32_t sB, const MmaChunks& c,
                                            bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < BK / 16; ++kk) {
    const uint64_t ad = sw128_desc(sA + kk * 32);
    const uint32_t acc = (accumulate || kk > 0) ? 1u : 0u;
    umma2_f16(tmem, ad, sw128_desc(sB + kk * 32), c.id0, acc);
    if (c.two) umma2_f16(tmem + 256u, ad, sw128_desc(sB + 128u * 128u + kk * 32), c.id1, acc);
  }
}

// ---------------------------------------------------------------------------
// Host: TMA descriptors
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D K-major map over a row-major [rows x k] half-precision matrix, box
// [box_rows x 64], 128-byte swizzle, zero fill outside the matrix.
inline bool make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t rows, int64_t k, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(k) * 2};
  cuuint32_t box[2] = {cuuint32_t(BK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType dt = dtype == DORA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace dora
