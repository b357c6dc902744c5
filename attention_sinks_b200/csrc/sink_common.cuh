// Shared definitions of the sink-cache kernels: launch arguments, the split plan that host
// and device both evaluate, PTX wrappers for mbarriers and bulk (TMA) copies, element
// conversions.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sinkb200 {

constexpr int kThreads = 128;                 // 4 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kPipeBytes = 98304;             // pipeline smem budget per CTA: 2 CTAs per SM
constexpr int kBarrierBytes = 128;            // mbarriers in front of the stages
constexpr int kSmemPerSM = 233472;            // B200: 228 KB shared memory per SM
constexpr int kSmemReservedPerCTA = 1024;
constexpr int kMaxSplits = 256;               // combine kernel keeps ns * G weights in smem
constexpr int kMaxGroup = 8;
// Clustered launches (every split of a pair in one thread-block cluster): at most this many
// splits (a non-portable cluster size), and a shift of at most kClusterHaloRows rows, whose
// halo rows each CTA stages in its own shared memory.
constexpr int kClusterMax = 16;
constexpr int kClusterHaloRows = 4;

__host__ __device__ inline int imin(int a, int b) { return a < b ? a : b; }
__host__ __device__ inline int imax(int a, int b) { return a > b ? a : b; }

// Arguments of one stream-kernel launch.  Output rows [row_begin, row_end) of every
// (batch, kv-head) pair are split into `ns` contiguous splits of `rows_per_split` rows.
// Output row r reads:
//   - buffer row r + drop (or the halo copy of it)  if drop > 0 and n_sink <= r < n_sink+window
//   - the new token (knew / vnew)                    if r == append_row
//   - buffer row r                                   otherwise (sinks, or drop == 0)
// and writes back (window rows when drop > 0, and the append row).
struct StreamArgs {
  char* kbuf;
  char* vbuf;
  int64_t k_sb, k_sh, v_sb, v_sh;  // element strides of batch / head; rows are contiguous
  const char* knew;
  const char* vnew;
  int64_t kn_sb, kn_sh, vn_sb, vn_sh;
  const char* q;
  int64_t q_sb, q_sh;
  char* out;
  int64_t o_sb, o_sh;
  const float* cos_tab;
  const float* sin_tab;
  int heads_kv, group;
  int n_sink, window, drop, rotate;
  int row_begin, row_end, append_row, written_end;
  int ns, rows_per_split, halo_rows;
  float scale_log2;
  const uint8_t* mask;  // optional [batch] x row_end booleans: attend to row r iff nonzero
  int64_t mask_sb;      // batch stride of the mask in bytes (0: one row shared by the batch)
  float* o_part;
  float* m_part;
  float* l_part;
  char* halo_k;
  char* halo_v;
  int* status;
  // 1: launched as clusters of ns CTAs along x (one cluster per pair).  Halo rows are then
  // staged in shared memory before a cluster barrier, and the split partials are merged
  // through distributed shared memory: no halo pre-pass, no combine kernel, no workspace
  // beyond the status word.
  int cluster;
  // Polls of each bounded mbarrier wait before it gives up (kWaitPolls unless a
  // failure-detection test shortens it).
  int wait_polls;
  // Failure-detection test hook, -1 when off: every CTA leaves its chunk `skip_chunk`
  // unissued (no copy, no arrival), so the wait for it runs out with nothing in flight.
  int skip_chunk;
  // Optional key copy in the value type (chunk steps): every output row r the launch handles
  // is also written, rounded to the value type, to kmirror row r (element strides of batch
  // and head km_sb / km_sh, rows contiguous).  NULL: none.
  char* kmirror;
  int64_t km_sb, km_sh;
};

// Rows [a, e) of split j.
__host__ __device__ inline void split_rows(int row_begin, int row_end, int rows_per_split, int j,
                                           int& a, int& e) {
  a = row_begin + j * rows_per_split;
  e = imin(a + rows_per_split, row_end);
}

// Source rows of the split of rows [a, e) that another split of the same launch may
// overwrite before this split reads them (none for the last split of a pair).  [hlo, hhi)
// in buffer-row space; empty when hlo >= hhi.  The split's window sources are
// [max(a, s) + drop, min(e, s + W) + drop); rows below e belong to the split itself (read
// before written, in order); rows from e up to `written_end` (exclusive) are destinations of
// later splits.
__host__ __device__ inline void halo_range(int n_sink, int window, int drop, int written_end,
                                           bool last, int a, int e, int& hlo, int& hhi) {
  hlo = hhi = 0;
  if (drop <= 0 || last) return;
  const int w0 = imax(a, n_sink), w1 = imin(e, n_sink + window);
  if (w0 >= w1) return;
  const int s0 = w0 + drop, s1 = w1 + drop;
  const int lo = imax(s0, e), hi = imin(s1, written_end);
  if (lo < hi) {
    hlo = lo;
    hhi = hi;
  }
}

// ------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Adds `bytes` to the transaction count the current phase waits for (no arrival).
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Default poll limit of a bounded wait: about a second with the back-off below.
constexpr int kWaitPolls = 1 << 20;

// Bounded wait for a phase of an mbarrier: false if the copies never landed (then the
// caller records SINK_STATUS_WAIT_TIMEOUT and abandons its work instead of hanging).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int polls = kWaitPolls) {
#pragma unroll 1
  for (int i = 0; i < polls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 64) __nanosleep(256);
  }
  return false;
}

// global -> shared bulk copy, completion counted on `bar` in bytes.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// shared -> global bulk copy, tracked by bulk groups.
__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's generic-proxy global stores before async-proxy (TMA) accesses that a
// later barrier makes depend on them.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start before its predecessor ends; grid_dependency_wait() blocks until the
// predecessor grid has completed and its memory is visible.  allow_dependents() lets the
// next kernel of the stream start launching.  Both are no-ops without the launch attribute.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Thread-block cluster: a hardware barrier over every thread of the cluster (release /
// acquire orders shared and global memory across its CTAs), and reads of another CTA's
// shared memory through the cluster window.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Split cluster barrier: arrive (release) and wait (acquire) as two steps, so a CTA can keep
// working between its arrival and the point where it needs the other CTAs' arrivals.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// ------------------------------------------------------------------ element conversions

template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
  static __device__ __forceinline__ void load4(const float* p, float (&o)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x;
    o[1] = v.y;
    o[2] = v.z;
    o[3] = v.w;
  }
  static __device__ __forceinline__ void store4(float* p, const float (&o)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(o[0], o[1], o[2], o[3]);
  }
  static __device__ __forceinline__ void load8(const float* p, float (&o)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    o[0] = a.x;
    o[1] = a.y;
    o[2] = a.z;
    o[3] = a.w;
    o[4] = b.x;
    o[5] = b.y;
    o[6] = b.z;
    o[7] = b.w;
  }
  // round-trip through the storage type (identity for float)
  static __device__ __forceinline__ float round(float x) { return x; }
};

template <>
struct Elem<__nv_bfloat16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ void load4(const T* p, float (&o)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    o[0] = a.x;
    o[1] = a.y;
    o[2] = b.x;
    o[3] = b.y;
  }
  static __device__ __forceinline__ void store4(T* p, const float (&o)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(o[0], o[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(o[2], o[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  }
  static __device__ __forceinline__ void load8(const T* p, float (&o)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
};

template <>
struct Elem<__half> {
  using T = __half;
  static __device__ __forceinline__ float to_f(T x) { return __half2float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ void load4(const T* p, float (&o)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    o[0] = a.x;
    o[1] = a.y;
    o[2] = b.x;
    o[3] = b.y;
  }
  static __device__ __forceinline__ void store4(T* p, const float (&o)[4]) {
    __half2 a = __floats2half2_rn(o[0], o[1]);
    __half2 b = __floats2half2_rn(o[2], o[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  }
  static __device__ __forceinline__ void load8(const T* p, float (&o)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};

// Shared memory the stream kernel's end-of-split merge reuses from its stages: the per-warp
// partials (m, l, acc per group).
__host__ __device__ constexpr int merge_scratch_bytes(int warps, int groups, int D) {
  return warps * groups * (D + 2) * 4;
}

// Floats of a clustered launch's merge area: the pair's G * D outputs split into ns equal
// slices, one slice per CTA, each received from every CTA (ns * ceil(G * D / ns) <=
// G * D + ns - 1 floats), then every CTA's (M, L) per group, and the merge weights.
__host__ __device__ constexpr int cluster_merge_floats(int groups, int D) {
  return groups * D + kClusterMax + 3 * groups * kClusterMax;
}

// Compile-time geometry of the stream kernel for one (K type, V type, head_dim).
//   LPR lanes share one cache row: lane i of a row owns K dims [4i, 4i+4) and
//   [D/2 + 4i, D/2 + 4i + 4) (the RoPE half-split partners) and V dims [8i, 8i + 8).
//   A warp covers RPW rows per step; a chunk of T rows is 4 steps of all 4 warps.
template <typename KT, typename VT, int D>
struct StreamGeom {
  static_assert(D == 64 || D == 128 || D == 256, "head_dim");
  static constexpr int LPR = D / 8;
  static constexpr int RPW = 32 / LPR;
  static constexpr int STEPS = 4;
  static constexpr int T = STEPS * kWarps * RPW;
  static constexpr int KROW = D * (int)sizeof(KT);
  static constexpr int VROW = D * (int)sizeof(VT);
  static constexpr int STAGE = T * (KROW + VROW);
  static constexpr int S0 = kPipeBytes / STAGE;
  static constexpr int S = S0 < 2 ? 2 : (S0 > 4 ? 4 : S0);
  static constexpr int HALO = kClusterHaloRows * (KROW + VROW);  // clustered launches' halo rows
  // clustered launches' merge area: the split partials other CTAs of the cluster push here
  static constexpr int MERGE = cluster_merge_floats(kMaxGroup, D) * 4;
  // what the split planner counts per CTA (CTAs per SM), and what a launch opts into
  static constexpr int PLAN_SMEM = kBarrierBytes + S * STAGE + HALO;
  static constexpr int SMEM = PLAN_SMEM + MERGE;
  // the end-of-split merge reuses the stage memory (merge_scratch_bytes)
  static_assert(merge_scratch_bytes(kWarps, kMaxGroup, D) <= S * STAGE, "merge scratch");
  static_assert(kBarrierBytes >= 8 * (S + 1), "stage barriers and the halo barrier");
};

}  // namespace sinkb200
