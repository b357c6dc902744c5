// Split-K decode attention on the 5th-generation tensor cores (tcgen05) for 16-bit K and V
// with head_dim 128: the attention of the ring-buffer (v2) step and of plain decode
// attention over model-dtype keys (src/sinkcache/decode_attention.py:29-130).
//
// Persistent: one CTA (192 threads; 256 with the place warps of a fused ring-buffer step)
// per SM (the pipeline takes 192 KB of shared memory)
// walks the work items (split, batch * kv-head) i = blockIdx.x, blockIdx.x + gridDim.x, ...
// (tc_item) as one continuous stream of 128-row key chunks, so the copy pipeline stays full
// across item boundaries.  Per chunk:
//   - TMA (cp.async.bulk.tensor, 4-D maps over [B, Hkv, slots, 128], 128-byte swizzle)
//     loads the chunk's K and V as two 64-column boxes each into one of 3 stages;
//   - one thread issues S^T = K . Q^T as 8 tcgen05.mma (M = 128 keys, N = 16 query rows of
//     which the first G are the GQA group, K = 16 dims each) into TMEM;
//   - thread i owns key i: it reads its G scores with tcgen05.ld, and the CTA runs the
//     online softmax (chunk max across the 4 warps, exp2 in the log2 domain, fp32);
//   - P (16-bit, [16 query rows][128 keys], swizzled like the TMA tiles) goes to shared
//     memory and one thread issues O^T = V^T . P^T as 8 tcgen05.mma (M = 128 dims, V read
//     MN-major straight from its TMA tile, N = 16, K = 16 keys each);
//   - O^T accumulates in TMEM across the item's chunks.  P is taken against a reference max
//     that only moves when a chunk's scores exceed it by more than 2^8 (then O^T is read,
//     rescaled and written back with tcgen05.ld/st): the common chunk needs no TMEM round
//     trip and one CTA barrier;
//   - S^T and P are double-buffered and the next chunk's S^T is issued before this chunk's
//     softmax, so the MMAs run under the softmax;
//   - O^T is double-buffered by item: an item's epilogue (thread d, TMEM lane d of O^T,
//     reads its G outputs) runs during the next item's first chunk, and the q rows of the
//     item after next are prefetched by TMA, so item boundaries cost no exposed latency.
// Results: the normalised output (one split) or fp32 partials (O, reference max, sum of P)
// in the layout the split combine kernel reads.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "sink_chunk.cuh"
#include "sink_v2.cuh"

namespace sinkb200 {

constexpr int kTcRows = 128;                       // keys per chunk (MMA M of S^T)
constexpr int kTcD = 128;                          // head_dim (MMA M of O^T)
constexpr int kTcStages = 3;
constexpr int kTcBoxBytes = 64 * kTcRows * 2;      // one TMA box: 64 columns x 128 rows, 16-bit
constexpr int kTcStageBytes = 4 * kTcBoxBytes;     // K box 0, K box 1, V box 0, V box 1
constexpr int kTcN = 16;                           // MMA N: query rows (GQA group, zero padded)
constexpr int kTcOperandBytes = 2 * kTcN * 128;    // Q or P: two 64-column boxes of 16 rows
// K ring | V ring | Q (three slots: items i, i+1, i+2) | P (two buffers) | barriers, reductions
constexpr int kTcQSlots = 3;
constexpr int kTcSmemBytes = 1024 + kTcStages * kTcStageBytes + (kTcQSlots + 2) * kTcOperandBytes + 512;
constexpr int kTcTmemCols = 64;  // S^T buffers at [0, 16) and [16, 32), O^T buffers at [32, 48) and [48, 64)
constexpr float kTcRescaleLog2 = 8.f;              // rescale O when a score passes the reference by 2^8

struct TcArgs {
  CUtensorMap kmap;       // [B, Hkv, slots, 128] keys, box {64, 128, 1, 1}, 128-byte swizzle
  CUtensorMap vmap;       // values, same geometry
  CUtensorMap qmap;       // [B, Hq, 128] queries, box {64, G, 1}, 128-byte swizzle (if q_async)
  const char* q;          // [B, Hq, 1, 128] in the cache dtype
  int64_t q_sb, q_sh;
  char* out;              // [B, 1, Hq, 128]
  int64_t o_sb, o_sh;
  const uint8_t* mask;    // optional [batch] x row_end booleans (attend iff nonzero)
  int64_t mask_sb;
  float* o_part;
  float* m_part;
  float* l_part;
  int* status;
  int heads_kv, group, row_end, rows_per_split, ns, pairs;
  int q_async;            // qmap is valid: each item's q rows are prefetched by TMA
  float scale_log2;
  // 1: one item per CTA and the ns CTAs of each pair launched as one cluster; the pair's
  // split partials are merged at the end of the kernel (no sink_combine_kernel launch).
  int cluster;
  // The ring-buffer step's place work in the same launch (the v2 decode step in one launch):
  // each CTA places the rows of its own items (no row belongs to two items) and the device
  // position advances as in sink_v2_place_kernel.  kTcPlaceFirst: every thread places
  // before the pipeline starts (short steps; items split-major, so that the pairs' region
  // and new-token items land on different CTAs).  kTcPlaceWarps: two warps place item by
  // item beside the pipeline, which holds back only the chunks holding placed rows (long
  // steps).  kTcPlaceNone: attention only.
  int place;
  V2PlaceArgs pa;
};

// Largest cluster (a pair's splits) for the in-cluster merge; sizes above 8 are used only
// where the device's occupancy query says every such cluster fits at once.
constexpr int kTcClusterMax = 16;

// ------------------------------------------------------------------ tcgen05 / TMA wrappers

// Shared-memory matrix descriptor, 128-byte swizzle (SM100 format, version 1).  K-major:
// rows of 128 bytes, 8-row groups 1024 bytes apart.  MN-major: 64-element column blocks
// `lbo` bytes apart, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo_bytes) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((lbo_bytes >> 4) & 0x3FFF) << 16) |
         (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulate, A and B both `fmt` (0 fp16, 1 bf16),
// A K-major or MN-major, B K-major, M = 128, N = 16.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t fmt, bool a_mn_major) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (uint32_t(a_mn_major) << 15) |
         (uint32_t(kTcN >> 3) << 17) | (uint32_t(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                       bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(uint32_t(accumulate))
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// N consecutive 32-bit TMEM columns of this thread's lane (warp w reads lanes 32w..32w+31).
template <int N>
__device__ __forceinline__ void tc_ld(uint32_t taddr, float (&v)[N]) {
  uint32_t r[8];
  if constexpr (N == 1) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(taddr));
  } else if constexpr (N == 2) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(taddr));
  } else if constexpr (N == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  } else {
    static_assert(N == 8, "1, 2, 4 or 8 columns");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  }
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = __uint_as_float(r[i]);
}

// Store N consecutive 32-bit TMEM columns of this thread's lane.
template <int N>
__device__ __forceinline__ void tc_st(uint32_t taddr, const float (&v)[N]) {
  uint32_t r[8];
#pragma unroll
  for (int i = 0; i < N; ++i) r[i] = __float_as_uint(v[i]);
  if constexpr (N == 1) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r[0]) : "memory");
  } else if constexpr (N == 2) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(r[0]), "r"(r[1])
                 : "memory");
  } else if constexpr (N == 4) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3])
                 : "memory");
  } else {
    static_assert(N == 8, "1, 2, 4 or 8 columns");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
  }
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int row,
                                            int h, int b, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(row), "r"(h), "r"(b), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Byte offset of element (row r < 16, column c < 128) of a Q or P operand: two boxes of 64
// columns, rows of 128 bytes, 16-byte chunks swizzled by the row (as TMA's 128-byte mode).
__device__ __forceinline__ uint32_t tc_operand_offset(int r, int c) {
  const int box = c >> 6, col = c & 63;
  return uint32_t(box * (kTcN * 128) + r * 128 + ((((col >> 3) ^ r) & 7) << 4) + (col & 7) * 2);
}

// ------------------------------------------------------------------ kernel

constexpr int kTcPlaceNone = 0, kTcPlaceFirst = 1, kTcPlaceWarps = 2;

// Item `it` = (split j, pair p): its (batch, head), rows [a, e) and chunk count.  Pair-major
// (it = p * ns + j); split-major (it = j * pairs + p) with kTcPlaceFirst, whose CTAs place
// before they load: the pairs' items over the same rows -- the last split's region rows,
// the split holding this step's ring slot -- are then consecutive and land on different
// CTAs.  A clustered launch (its clusters are the pairs) is always pair-major.
struct TcItem {
  int p, j, b, h, a, e, n;
};

__device__ __forceinline__ TcItem tc_item(const TcArgs& A, int it) {
  TcItem w;
  if (A.cluster || A.place != kTcPlaceFirst) {
    w.p = it / A.ns;
    w.j = it - w.p * A.ns;
  } else {
    w.j = it / A.pairs;
    w.p = it - w.j * A.pairs;
  }
  w.b = w.p / A.heads_kv;
  w.h = w.p - w.b * A.heads_kv;
  split_rows(0, A.row_end, A.rows_per_split, w.j, w.a, w.e);
  w.n = (w.e - w.a + kTcRows - 1) / kTcRows;
  return w;
}

// Q of item w (G rows of 128 dims, unscaled) into an operand slot; rows past G are zeros.
// 16-bit loads: no alignment is asked of q.
template <typename T>
__device__ __forceinline__ void tc_load_q(const TcArgs& A, const TcItem& w, unsigned char* slot) {
  const int G = A.group;
  const T* qb = reinterpret_cast<const T*>(A.q) + w.b * A.q_sb + int64_t(w.h) * G * A.q_sh;
  for (int i = threadIdx.x; i < kTcN * 16; i += kThreads) {
    const int r = i >> 4, c = (i & 15) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < G) {
      const uint16_t* src = reinterpret_cast<const uint16_t*>(qb + r * A.q_sh + c);
      uint16_t e[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = src[k];
      v = make_uint4(e[0] | (uint32_t(e[1]) << 16), e[2] | (uint32_t(e[3]) << 16),
                     e[4] | (uint32_t(e[5]) << 16), e[6] | (uint32_t(e[7]) << 16));
    }
    *reinterpret_cast<uint4*>(slot + tc_operand_offset(r, c)) = v;
  }
}

// Warp roles: warps 0-3 run the softmax and the epilogues (thread i <-> TMEM lane i), warp 4
// issues the MMAs, warp 5 issues the TMA loads.  They hand work to each other through
// mbarriers only, so loads run up to three chunks ahead and MMA issue overlaps the softmax.
// Warps 6-7 do the ring-buffer step's place work under kTcPlaceWarps and publish their
// progress through release/acquire flags in shared memory; the load warp holds back only
// the chunks that contain rows they write.
constexpr int kTcMmaWarp = 4, kTcLoadWarp = 5, kTcPlaceWarp = 6;
constexpr int kTcPlaceThreads = 64;
// Threads of a launch: the six pipeline warps, plus the two place warps when PW (the
// kTcPlaceWarps instantiation; a CTA that never places carries no idle warps).
__host__ __device__ constexpr int tc_threads(bool pw) { return 32 * kTcPlaceWarp + (pw ? kTcPlaceThreads : 0); }

__device__ __forceinline__ void tc_place_sync() {  // the place warps only
  asm volatile("barrier.cta.sync 2, %0;" ::"n"(kTcPlaceThreads) : "memory");
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}
// Waits (bounded, like mbar_wait_bounded) until *p >= target; false when it gave up.
__device__ __forceinline__ bool wait_flag_bounded(const uint32_t* p, uint32_t target) {
  const uint32_t a = smem_addr(p);
  for (int i = 0; i < kWaitPolls; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    if (v >= target) return true;
    __nanosleep(32);
  }
  return false;
}

__device__ __forceinline__ bool tc_softmax_or(bool pred) {  // OR over the 128 softmax threads
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(pred))
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void tc_softmax_sync() { asm volatile("barrier.cta.sync 1, 128;" ::: "memory"); }

template <typename T, int GMAX, bool PW>
__global__ void __launch_bounds__(tc_threads(PW), 1) sink_attend_tc_kernel(const __grid_constant__ TcArgs A) {
  constexpr int kTcThreads = tc_threads(PW);
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles want 1024-byte alignment
  unsigned char* gbase = smem_raw + (base - raw);
  const uint32_t kring = base, vring = base + kTcStages * 2 * kTcBoxBytes;
  const uint32_t s_q = base + kTcStages * kTcStageBytes;  // kTcQSlots Q slots
  const uint32_t s_p = s_q + kTcQSlots * kTcOperandBytes; // two P buffers
  const uint32_t s_bar = s_p + 2 * kTcOperandBytes;
  // mbarriers (8 bytes each): kfull, vfull, kempty, vempty [kTcStages]; qfull, qempty
  // [kTcQSlots]; sready, pready [2]
  const uint32_t bar_kfull = s_bar, bar_vfull = bar_kfull + 8 * kTcStages;
  const uint32_t bar_kempty = bar_vfull + 8 * kTcStages, bar_vempty = bar_kempty + 8 * kTcStages;
  const uint32_t bar_qfull = bar_vempty + 8 * kTcStages, bar_qempty = bar_qfull + 8 * kTcQSlots;
  const uint32_t bar_sready = bar_qempty + 8 * kTcQSlots, bar_pready = bar_sready + 16;
  const uint32_t bar_mdone = bar_pready + 16;  // every MMA the MMA warp issued has completed
  unsigned char* q_g = gbase + (s_q - base);
  unsigned char* p_g = gbase + (s_p - base);
  float* red = reinterpret_cast<float*>(gbase + (s_bar - base) + 192);  // [4 warps][8]: chunk max
  float* red2 = red + 32;                                               // [4 warps][8]: item sums
  int* flag = reinterpret_cast<int*>(red2 + 32);                        // CTA failure flag
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red2 + 40);
  long long* t_s = reinterpret_cast<long long*>(red2 + 42);             // place: the position t
  // kTcPlaceWarps progress: [0] t published, [1] 1 + the last item ord whose rows are placed
  uint32_t* pflags = reinterpret_cast<uint32_t*>(red2 + 44);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = A.group;
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescQK = tc_idesc(kFmt, false);
  constexpr uint32_t kIdescPV = tc_idesc(kFmt, true);
  const int items = A.ns * A.pairs;
  const int my_items = int(blockIdx.x) < items ? (items - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
  auto item_of = [&](int ord) { return tc_item(A, int(blockIdx.x) + ord * int(gridDim.x)); };

  // ---- set-up (reads no global memory: overlaps the predecessor's tail)
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(bar_kfull + 8 * s, 1);
      mbar_init(bar_vfull + 8 * s, 1);
      mbar_init(bar_kempty + 8 * s, 1);
      mbar_init(bar_vempty + 8 * s, 1);
    }
#pragma unroll
    for (int s = 0; s < kTcQSlots; ++s) {
      mbar_init(bar_qfull + 8 * s, 1);
      mbar_init(bar_qempty + 8 * s, 1);
    }
    mbar_init(bar_sready, 1);
    mbar_init(bar_sready + 8, 1);
    mbar_init(bar_pready, kThreads);
    mbar_init(bar_pready + 8, kThreads);
    mbar_init(bar_mdone, 1);
    *flag = 0;
    pflags[0] = pflags[1] = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Operand rows past the group stay zero for the whole kernel (Q slots and P buffers).
  for (int i = tid; i < (kTcQSlots + 2) * kTcN * 16; i += kTcThreads) {
    const int buf = i / (kTcN * 16), r = (i >> 4) & (kTcN - 1), c = (i & 15) * 8;
    if (r >= G)
      *reinterpret_cast<uint4*>(q_g + buf * kTcOperandBytes + tc_operand_offset(r, c)) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();  // the MMAs read these rows through the async proxy
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto tmem_o = [&](int item_ord) { return tmem + 2 * kTcN + (item_ord & 1) * kTcN; };

  grid_dependency_wait();  // the producers of q and of the cache rows are complete

  if (A.place == kTcPlaceFirst) {  // every thread, before the pipeline starts
    if (tid == 0) *t_s = A.pa.position ? A.pa.position[0] : A.pa.t_host;
    __syncthreads();
    const long long t = *t_s;
    const long long ws = v2_window_start(A.pa, t);
    for (int ord = 0; ord < my_items; ++ord) {
      const TcItem w = item_of(ord);
      v2_place_pair<T, kTcD>(A.pa, w.b, w.h, t, ws, w.a, w.e, tid, kTcThreads);
    }
    fence_proxy_async_global();  // the TMA loads below read the placed rows
    __syncthreads();
    if (tid == 0 && A.pa.position) v2_position_arrive(A.pa, t);  // every CTA has read t
  }

  // kTcPlaceWarps: rows [a, e) of an item that the place warps write (the new token's ring
  // slot, region rows)
  auto slot_in = [&](long long r, const TcItem& w) { return A.pa.knew != nullptr && w.a <= r && r < w.e; };
  auto region_in = [&](int lo, int hi) { return A.pa.R > 0 && hi > A.pa.ring && lo < A.pa.ring + A.pa.R; };

  bool failed = false;
  if (warp == kTcLoadWarp) {
    // ================================================================ TMA loads (one lane)
    if (lane == 0 && my_items > 0) {
      // kTcPlaceWarps: the ring slot this step writes
      const bool warps_place = PW && A.place == kTcPlaceWarps;
      long long new_row = -1;
      if (warps_place) {
        if (!wait_flag_bounded(pflags, 1)) failed = true;
        new_row = (*t_s - A.pa.n_sink) % A.pa.ring;
        if (new_row < 0) new_row += A.pa.ring;
      }
      int seq = 0;
      for (int ord = 0; ord < my_items && !failed; ++ord) {
        const TcItem w = item_of(ord);
        bool placed = !warps_place;  // this item's placed rows are written
        const int qs = ord % kTcQSlots;
        if (A.q_async && ord >= kTcQSlots &&
            !mbar_wait_bounded(bar_qempty + 8 * qs, ((ord / kTcQSlots) - 1) & 1)) {
          failed = true;
          break;
        }
        if (A.q_async) {
          const uint32_t dst = s_q + qs * kTcOperandBytes, bar = bar_qfull + 8 * qs;
          mbar_arrive_expect_tx(bar, 2 * G * 128);
          tma_load_3d(dst, &A.qmap, 0, w.h * G, w.b, bar);
          tma_load_3d(dst + kTcN * 128, &A.qmap, 64, w.h * G, w.b, bar);
        }
        for (int c = 0; c < w.n; ++c, ++seq) {
          const int slot = seq % kTcStages, use = seq / kTcStages;
          const int row = w.a + c * kTcRows;
          const int rend = imin(row + kTcRows, w.e);
          if (!placed && (region_in(row, rend) || (A.pa.knew != nullptr && row <= new_row && new_row < rend))) {
            if (!wait_flag_bounded(pflags + 1, uint32_t(ord) + 1)) {  // this chunk holds placed rows
              failed = true;
              break;
            }
            placed = true;
          }
          if (seq >= kTcStages && !mbar_wait_bounded(bar_kempty + 8 * slot, (use - 1) & 1)) {
            failed = true;
            break;
          }
          uint32_t dst = kring + slot * (2 * kTcBoxBytes), bar = bar_kfull + 8 * slot;
          mbar_arrive_expect_tx(bar, 2 * kTcBoxBytes);
          tma_load_4d(dst, &A.kmap, 0, row, w.h, w.b, bar);
          tma_load_4d(dst + kTcBoxBytes, &A.kmap, 64, row, w.h, w.b, bar);
          if (seq >= kTcStages && !mbar_wait_bounded(bar_vempty + 8 * slot, (use - 1) & 1)) {
            failed = true;
            break;
          }
          dst = vring + slot * (2 * kTcBoxBytes);
          bar = bar_vfull + 8 * slot;
          mbar_arrive_expect_tx(bar, 2 * kTcBoxBytes);
          tma_load_4d(dst, &A.vmap, 0, row, w.h, w.b, bar);
          tma_load_4d(dst + kTcBoxBytes, &A.vmap, 64, row, w.h, w.b, bar);
        }
      }
      if (failed) {  // let the copies in flight land before the CTA can exit (bounded waits)
        for (int i = seq - 1; i >= 0 && i >= seq - kTcStages; --i) {
          mbar_wait_bounded(bar_kfull + 8 * (i % kTcStages), (i / kTcStages) & 1);
          mbar_wait_bounded(bar_vfull + 8 * (i % kTcStages), (i / kTcStages) & 1);
        }
      }
    }
  } else if (warp == kTcMmaWarp) {
    // ================================================================ MMA issue (one lane)
    if (lane == 0 && my_items > 0) {
      // S^T = K . Q^T for chunk `seq` (item `ord`, chunk `c` of `n`)
      auto qk = [&](int seq, int ord, int c, int n) -> bool {
        const int slot = seq % kTcStages, qs = ord % kTcQSlots;
        if (c == 0 && A.q_async && !mbar_wait_bounded(bar_qfull + 8 * qs, (ord / kTcQSlots) & 1)) return false;
        if (!mbar_wait_bounded(bar_kfull + 8 * slot, (seq / kTcStages) & 1)) return false;
        const uint32_t sb = kring + slot * (2 * kTcBoxBytes), qb = s_q + qs * kTcOperandBytes;
        const uint32_t d = tmem + (seq & 1) * kTcN;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTcD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kTcBoxBytes + (kk & 3) * 32;
          const uint32_t qoff = (kk >> 2) * (kTcN * 128) + (kk & 3) * 32;
          tc_mma(d, tc_desc(sb + off, 16), tc_desc(qb + qoff, 16), kIdescQK, kk > 0);
        }
        tc_commit(bar_sready + 8 * (seq & 1));
        tc_commit(bar_kempty + 8 * slot);
        if (c + 1 == n) tc_commit(bar_qempty + 8 * qs);
        return true;
      };
      int seq = 0;
      TcItem w = item_of(0), wn = w;
      int ord = 0, c = 0;
      if (!qk(0, 0, 0, w.n)) failed = true;
      while (!failed && ord < my_items) {
        // the next chunk's S^T first, so the tensor pipe works under this chunk's softmax
        int nord = ord, nc = c + 1;
        wn = w;
        if (nc == w.n) {
          nc = 0;
          ++nord;
          if (nord < my_items) wn = item_of(nord);
        }
        if (nord < my_items && !qk(seq + 1, nord, nc, nc == 0 ? wn.n : w.n)) {
          failed = true;
          break;
        }
        // O^T (+)= V^T . P^T once the softmax warps have written P (and rescaled O^T)
        const int slot = seq % kTcStages;
        if (!mbar_wait_bounded(bar_pready + 8 * (seq & 1), (seq >> 1) & 1) ||
            !mbar_wait_bounded(bar_vfull + 8 * slot, (seq / kTcStages) & 1)) {
          failed = true;
          break;
        }
        const uint32_t vb = vring + slot * (2 * kTcBoxBytes), pb = s_p + (seq & 1) * kTcOperandBytes;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kTcRows / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * (kTcN * 128) + (kk & 3) * 32;
          tc_mma(tmem_o(ord), tc_desc(vb + kk * 2048, kTcBoxBytes), tc_desc(pb + poff, 16), kIdescPV,
                 !(c == 0 && kk == 0));
        }
        tc_commit(bar_vempty + 8 * slot);
        ++seq;
        ord = nord;
        c = nc;
        w = wn;
      }
      tc_commit(bar_mdone);  // TMEM is freed only after every MMA has completed
      mbar_wait_bounded(bar_mdone, 0);
    }
  } else if (PW && warp >= kTcPlaceWarp) {
    // ================================================================ place work (2 warps)
    // kTcPlaceWarps: the ring-buffer step's state update for the rows of this CTA's items,
    // item by item in the order the loads reach them (t published first).  Each item's
    // generic stores are ordered before the loads' async-proxy reads of them by the writers'
    // proxy fence, the place barrier and a release store the load warp acquires.
    if (A.place == kTcPlaceWarps) {
      const int ptid = tid - 32 * kTcPlaceWarp;
      if (ptid == 0) {
        *t_s = A.pa.position ? A.pa.position[0] : A.pa.t_host;
        st_release_u32(pflags, 1);
      }
      tc_place_sync();
      const long long t = *t_s;
      const long long ws = v2_window_start(A.pa, t);
      long long new_row = (t - A.pa.n_sink) % A.pa.ring;
      if (new_row < 0) new_row += A.pa.ring;
      for (int ord = 0; ord < my_items; ++ord) {
        const TcItem w = item_of(ord);
        if (!slot_in(new_row, w) && !region_in(w.a, w.e)) continue;
        v2_place_pair<T, kTcD>(A.pa, w.b, w.h, t, ws, w.a, w.e, ptid, kTcPlaceThreads);
        fence_proxy_async_global();
        tc_place_sync();
        if (ptid == 0) st_release_u32(pflags + 1, uint32_t(ord) + 1);
      }
      // every CTA has read t before it counts itself in; the last stores t + 1
      if (ptid == 0 && A.pa.position) v2_position_arrive(A.pa, t);
    }
  } else {
    // ================================================================ softmax (4 warps)
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    if (!A.q_async) {  // q rows not 16-byte aligned: these warps stage Q with plain loads
      if (my_items > 0) tc_load_q<T>(A, item_of(0), q_g);
      if (my_items > 1) tc_load_q<T>(A, item_of(1), q_g + kTcOperandBytes);
      fence_proxy_async_smem();
      tc_softmax_sync();
      if (tid == 0) {
        if (my_items > 0) mbar_arrive(bar_qfull);
        if (my_items > 1) mbar_arrive(bar_qfull + 8);
      }
    }
    float mref[GMAX], l[GMAX], l_prev[GMAX], m_prev[GMAX];
    TcItem cur = my_items > 0 ? item_of(0) : TcItem{}, prev = cur;
    int prev_last = -1;
    auto reduce_l_prev = [&]() {
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        float sm = l_prev[g];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sm += __shfl_xor_sync(kFull, sm, off);
        if (lane == 0) red2[warp * 8 + g] = sm;
      }
    };
    auto write_item = [&](int pord) {  // after red2 holds the warps' sums of l_prev
      if (!mbar_wait_bounded(bar_vempty + 8 * (prev_last % kTcStages), (prev_last / kTcStages) & 1)) failed = true;
      float o[GMAX];
      __syncwarp();
      tc_fence_after();
      tc_ld<GMAX>(tmem_o(pord) + lane_base, o);
      tc_wait_ld();
      tc_fence_before();
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        if (g >= G || failed) break;
        const float L = red2[g] + red2[8 + g] + red2[16 + g] + red2[24 + g];
        const int d = tid;  // output dim owned by this thread (TMEM lane of O^T)
        if (A.ns == 1) {
          T* out = reinterpret_cast<T*>(A.out) + prev.b * A.o_sb + (prev.h * G + g) * A.o_sh;
          out[d] = Elem<T>::from_f(L > 0.f ? o[g] / L : 0.f);
        } else {
          const size_t part = (size_t(prev.p) * A.ns + prev.j) * G + g;
          A.o_part[part * kTcD + d] = o[g];
          if (d == 0) {
            A.m_part[part] = m_prev[g];
            A.l_part[part] = L;
          }
        }
      }
    };

    int ord = 0, chunk = 0;
#pragma unroll 1
    for (int seq = 0; ord < my_items; ++seq) {
      const bool first = chunk == 0;
      const bool last_in_item = chunk + 1 == cur.n;
      if (first) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          mref[g] = kNegInf;
          l[g] = 0.f;
        }
      }
      if (!failed && !mbar_wait_bounded(bar_sready + 8 * (seq & 1), (seq >> 1) & 1)) failed = true;
      float s[GMAX];
      __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the divergent waits
      tc_fence_after();
      tc_ld<GMAX>(tmem + (seq & 1) * kTcN + lane_base, s);
      tc_wait_ld();
      tc_fence_before();
      if (first && ord > 0) reduce_l_prev();
      // plain-load path: item ord + 2's Q goes to the slot item ord - 1 used (its S^T MMAs,
      // all issued before this chunk's, have completed)
      const bool stage_q = !A.q_async && first && ord + 2 < my_items;
      if (stage_q) tc_load_q<T>(A, item_of(ord + 2), q_g + ((ord + 2) % kTcQSlots) * kTcOperandBytes);
      const int row = cur.a + chunk * kTcRows + tid;
      const uint8_t* mrow = A.mask != nullptr ? A.mask + cur.b * A.mask_sb : nullptr;
      const bool valid = row < cur.e && (mrow == nullptr || mrow[row] != 0);
      bool need = false;
      unsigned char* pbuf = p_g + (seq & 1) * kTcOperandBytes;
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        s[g] = (valid && g < G) ? s[g] * A.scale_log2 : kNegInf;
        need |= s[g] > mref[g] + kTcRescaleLog2;
      }
      float pfast[GMAX];  // P against the current reference: kept only if no thread needs a rescale
      if (!need) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          pfast[g] = s[g] == kNegInf ? 0.f : exp2f(s[g] - mref[g]);
          if (g < G) *reinterpret_cast<T*>(pbuf + tc_operand_offset(g, tid)) = Elem<T>::from_f(pfast[g]);
        }
      }
      if (stage_q) fence_proxy_async_smem();
      // a failed wait takes the (uniform) slow path, where the failure is agreed on
      const bool any_need = tc_softmax_or(need || failed);
      if (stage_q && tid == 0) mbar_arrive(bar_qfull + 8 * ((ord + 2) % kTcQSlots));
      if (first && ord > 0) write_item(ord - 1);  // the previous item's output, off the MMA path
      if (!any_need) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) l[g] += pfast[g];
      } else {
        // ---- slow path: move the reference max up to this chunk's max
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          float mx = s[g];
#pragma unroll
          for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
          if (lane == 0) red[warp * 8 + g] = mx;
        }
        tc_softmax_sync();
        float alpha[GMAX];
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          const float cm = fmaxf(fmaxf(red[g], red[8 + g]), fmaxf(red[16 + g], red[24 + g]));
          const float mn = fmaxf(mref[g], cm);
          alpha[g] = (mref[g] == kNegInf || mn == kNegInf) ? 0.f : exp2f(mref[g] - mn);
          mref[g] = mn;
        }
        if (!first) {  // O^T holds earlier chunks of this item: once they are in, rescale it
          const int pc = seq - 1;
          if (!mbar_wait_bounded(bar_vempty + 8 * (pc % kTcStages), (pc / kTcStages) & 1)) failed = true;
          float o[GMAX];
          __syncwarp();
          tc_fence_after();
          tc_ld<GMAX>(tmem_o(ord) + lane_base, o);
          tc_wait_ld();
#pragma unroll
          for (int g = 0; g < GMAX; ++g) o[g] *= alpha[g];
          tc_st<GMAX>(tmem_o(ord) + lane_base, o);
          tc_wait_st();
        }
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          const float pg = (s[g] == kNegInf || mref[g] == kNegInf) ? 0.f : exp2f(s[g] - mref[g]);
          l[g] = l[g] * alpha[g] + pg;
          if (g < G) *reinterpret_cast<T*>(pbuf + tc_operand_offset(g, tid)) = Elem<T>::from_f(pg);
        }
        failed = tc_softmax_or(failed);  // also keeps red until every thread has read it
        if (failed) break;               // uniform: every softmax thread leaves together
      }
      // (a failure in write_item above reaches the next chunk's barrier through need || failed)
      // P of this chunk (and any rescale of O^T) are complete: hand them to the MMA warp
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(bar_pready + 8 * (seq & 1));
      if (last_in_item) {
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          l_prev[g] = l[g];
          m_prev[g] = mref[g];
        }
        prev = cur;
        prev_last = seq;
        chunk = 0;
        if (++ord < my_items) cur = item_of(ord);
      } else {
        ++chunk;
      }
    }
    failed = tc_softmax_or(failed);  // uniform before the epilogue's barrier
    if (!failed && my_items > 0) {  // the last item's epilogue
      reduce_l_prev();
      tc_softmax_sync();
      write_item(my_items - 1);
    }
  }
  if (failed) atomicOr(flag, 1);
  allow_dependents();
  tc_fence_before();
  __syncthreads();
  if (*flag != 0 && tid == 0) atomicOr(A.status, 1);
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols)
                 : "memory");
  }
  if (A.cluster) {
    // Every CTA of the cluster has written its partial (the barrier's release/acquire makes
    // them visible); each merges a slice of the pair's G * 128 outputs, as the combine
    // kernel would.  Partials are read through L2 (.cg).
    cluster_sync();
    const int ns = A.ns;
    const int p = int(blockIdx.x) / ns, j = int(blockIdx.x) - p * ns;
    const int b = p / A.heads_kv, h = p - b * A.heads_kv;
    const size_t pb = size_t(p) * ns;
    // The K ring is idle now: per group, the ns partials' maxima and sums (loaded in
    // parallel, one per thread), turned into normalised weights by one warp per group.
    float* wts = reinterpret_cast<float*>(gbase);  // [GMAX][kTcClusterMax]
    float* mxs = wts + GMAX * kTcClusterMax;
    for (int t = tid; t < G * ns; t += kTcThreads) {
      const int g = t / ns, s = t - g * ns;
      mxs[g * kTcClusterMax + s] = __ldcg(A.m_part + (pb + s) * G + g);
      wts[g * kTcClusterMax + s] = __ldcg(A.l_part + (pb + s) * G + g);
    }
    __syncthreads();
    for (int g = warp; g < G; g += kTcThreads / 32) {  // one warp per group, one split per lane
      const bool live = lane < ns;
      const float w = split_weight(live ? mxs[g * kTcClusterMax + lane] : kNegInf,
                                   live ? wts[g * kTcClusterMax + lane] : 0.f);
      __syncwarp();
      if (live) wts[g * kTcClusterMax + lane] = w;
    }
    __syncthreads();
    // this CTA's equal slice of the pair's G * 128 outputs; an output's ns partials are
    // all requested before any is used
    const int per = (G * kTcD + ns - 1) / ns;
    const int lo = j * per, hi = imin(lo + per, G * kTcD);
    for (int idx = lo + tid; idx < hi; idx += kTcThreads) {
      const int g = idx / kTcD, d = idx - g * kTcD;
      float o_s[kTcClusterMax];
#pragma unroll
      for (int s = 0; s < kTcClusterMax; ++s)
        o_s[s] = s < ns ? __ldcg(A.o_part + ((pb + s) * G + g) * kTcD + d) : 0.f;
      float o = 0.f;
#pragma unroll
      for (int s = 0; s < kTcClusterMax; ++s)
        if (s < ns) o = __fmaf_rn(wts[g * kTcClusterMax + s], o_s[s], o);
      T* op = reinterpret_cast<T*>(A.out) + b * A.o_sb + (h * G + g) * A.o_sh;
      op[d] = Elem<T>::from_f(o);
    }
  }
}

}  // namespace sinkb200
