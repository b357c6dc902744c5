// Kernels of the sink-cache decode path.
//
//   sink_stream_kernel   one (split, batch * kv-head) work item per CTA: row chunks of the
//                        split are bulk-copied (TMA) into a shared-memory pipeline, window
//                        keys are re-rotated in fp32 registers and written back with bulk
//                        stores, and (ATTEND) a GQA online-softmax decode attention runs over
//                        the same rows.  With drop == 0 and no append row it is a plain
//                        split-K decode attention; with ATTEND == false a plain eviction.
//                        Launched as one cluster per pair (StreamArgs::cluster), it stages
//                        its halo rows in shared memory and merges the split partials
//                        across the cluster itself: the whole step in one launch.
//   sink_halo_kernel     copies the source rows a later split overwrites before an earlier
//                        split reads them (pre-pass of an unclustered in-place shift).
//   sink_combine_kernel  merges the per-split softmax partials (unclustered launches).
//   sink_append_kernel   writes new K/V rows (unfused path).
#pragma once

#include "sink_chunk.cuh"

namespace sinkb200 {

// Bulk-copy the sources of output rows [x, xe) of one (batch, head) into a stage: up to
// four contiguous segments (unshifted rows below the window; window rows shifted by drop,
// read directly below the halo range, from the halo copy `hk`/`hv` (row hlo first), and
// directly above it).  With no halo copy given, rows whose source lies in [hlo, hhi) are
// left for the caller to fill.  The append row is filled by threads.  Each segment adds its
// bytes to the stage barrier's expected count before its copies are issued, and one
// arrival at the end lets the phase complete once every byte has landed.
template <typename KT, typename VT, int D>
__device__ __forceinline__ void issue_rows(const StreamArgs& A, const KT* kb, const VT* vb, int x,
                                           int xe, int hlo, int hhi, const unsigned char* hk,
                                           const unsigned char* hv, uint32_t sk, uint32_t sv,
                                           uint32_t bar) {
  constexpr int KROW = D * (int)sizeof(KT), VROW = D * (int)sizeof(VT);
  auto segment = [&](int t, int n, const void* k, const void* v) {
    mbar_expect_tx(bar, uint32_t(n) * (KROW + VROW));
    bulk_g2s(sk + t * KROW, k, uint32_t(n) * KROW, bar);
    bulk_g2s(sv + t * VROW, v, uint32_t(n) * VROW, bar);
  };
  const int lowlim = A.drop > 0 ? A.n_sink : (A.append_row >= 0 ? A.append_row : A.row_end);
  const int p1 = imin(xe, lowlim);
  if (x < p1) segment(0, p1 - x, kb + size_t(x) * D, vb + size_t(x) * D);
  if (A.drop > 0) {
    const int w0 = imax(x, A.n_sink), w1 = imin(xe, A.n_sink + A.window);
    if (w0 < w1) {
      const int s0 = w0 + A.drop, s1 = w1 + A.drop;
      const bool halo = hlo < hhi;
      const int d1 = halo ? imin(s1, hlo) : s1;
      if (s0 < d1) segment(s0 - A.drop - x, d1 - s0, kb + size_t(s0) * D, vb + size_t(s0) * D);
      if (halo) {
        const int h0 = imax(s0, hlo), h1 = imin(s1, hhi);
        if (hk != nullptr && h0 < h1)
          segment(h0 - A.drop - x, h1 - h0, hk + size_t(h0 - hlo) * KROW, hv + size_t(h0 - hlo) * VROW);
        const int u0 = imax(s0, hhi);
        if (u0 < s1) segment(u0 - A.drop - x, s1 - u0, kb + size_t(u0) * D, vb + size_t(u0) * D);
      }
    }
  }
  mbar_arrive(bar);
}

// Rows of [x, xe) this step writes back: window rows (drop > 0) and the append row.
__device__ __forceinline__ void store_range(const StreamArgs& A, int x, int xe, int& lo, int& hi) {
  lo = hi = 0;
  if (A.drop > 0) {
    lo = imax(x, A.n_sink);
    hi = imin(xe, A.n_sink + A.window + (A.append_row >= 0 ? 1 : 0));
  } else if (A.append_row >= 0) {
    lo = imax(x, A.append_row);
    hi = imin(xe, A.append_row + 1);
  }
}

// The new token's K/V row into stage row t (converted to the key storage type).
template <typename KT, typename VT, int D, int NT = kThreads>
__device__ __forceinline__ void fill_append_row(const StreamArgs& A, int b, int h, KT* sk, VT* sv, int t) {
  const VT* kn = reinterpret_cast<const VT*>(A.knew) + b * A.kn_sb + h * A.kn_sh;
  const VT* vn = reinterpret_cast<const VT*>(A.vnew) + b * A.vn_sb + h * A.vn_sh;
  for (int d = threadIdx.x; d < D; d += NT) {
    sk[t * D + d] = Elem<KT>::from_f(Elem<VT>::to_f(kn[d]));
    sv[t * D + d] = vn[d];
  }
}

// Copy n rows (K and V) between shared-memory row arrays, 16 bytes per thread-step.
template <int KROW, int VROW, int NT = kThreads>
__device__ __forceinline__ void copy_rows(unsigned char* dk, unsigned char* dv, const unsigned char* sk,
                                          const unsigned char* sv, int n) {
  const int nk = n * KROW / 16, nv = n * VROW / 16;
  for (int i = threadIdx.x; i < nk; i += NT)
    reinterpret_cast<uint4*>(dk)[i] = reinterpret_cast<const uint4*>(sk)[i];
  for (int i = threadIdx.x; i < nv; i += NT)
    reinterpret_cast<uint4*>(dv)[i] = reinterpret_cast<const uint4*>(sv)[i];
}

// ============================================================================ split

// NW warps per CTA (4; 8 for clustered launches, where a CTA is usually alone on its SM and
// its chunk latency, not memory, bounds the step).
template <typename KT, typename VT, int D, int GMAX, bool ATTEND, int NW>
__global__ void __launch_bounds__(32 * NW) sink_stream_kernel(const __grid_constant__ StreamArgs A) {
  constexpr int NT = 32 * NW;
  using Gm = StreamGeom<KT, VT, D>;
  using Lanes = StreamLanes<KT, VT, D, GMAX, ATTEND, NW>;
  static_assert(merge_scratch_bytes(NW, GMAX, D) <= Gm::S * Gm::STAGE, "merge scratch");
  constexpr int T = Gm::T, S = Gm::S, KROW = Gm::KROW, STAGE = Gm::STAGE;
  constexpr int VROW = Gm::VROW;

  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t bar0 = smem_addr(smem);
  unsigned char* stages = smem + kBarrierBytes;
  unsigned char* halo_sk = stages + S * STAGE;  // clustered: this split's halo rows
  unsigned char* halo_sv = halo_sk + kClusterHaloRows * KROW;
  const uint32_t halo_bar = bar0 + 8 * S;
  const bool clustered = A.cluster != 0;  // grid-uniform

  grid_dependency_wait();  // halo copies (or the producers of q, k, v) complete
  const int tid = threadIdx.x;
  const int j = blockIdx.x, p = blockIdx.y;
  const int b = p / A.heads_kv, h = p - b * A.heads_kv;

  int a, e;
  split_rows(A.row_begin, A.row_end, A.rows_per_split, j, a, e);
  int hlo, hhi;
  halo_range(A.n_sink, A.window, A.drop, A.written_end, j >= A.ns - 1, a, e, hlo, hhi);
  const bool has_halo = hlo < hhi;

  KT* kb = reinterpret_cast<KT*>(A.kbuf) + b * A.k_sb + h * A.k_sh;
  VT* vb = reinterpret_cast<VT*>(A.vbuf) + b * A.v_sb + h * A.v_sh;
  const size_t halo_row0 = (size_t(p) * A.ns + j) * A.halo_rows;
  // Unclustered: halo rows come from the workspace copy made by sink_halo_kernel.
  // Clustered: issue_rows leaves them out and the consumer copies them from halo_sk/halo_sv.
  const unsigned char* hk =
      clustered ? nullptr : reinterpret_cast<const unsigned char*>(A.halo_k) + halo_row0 * KROW;
  const unsigned char* hv =
      clustered ? nullptr : reinterpret_cast<const unsigned char*>(A.halo_v) + halo_row0 * VROW;
  const int nchunks = (e - a + T - 1) / T;
  VT* kmir = A.kmirror != nullptr ? reinterpret_cast<VT*>(A.kmirror) + b * A.km_sb + h * A.km_sh : nullptr;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    mbar_init(halo_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // Chunks whose loads thread 0 has issued, and chunks whose arrival it has seen: on a
  // failure, the loads in between are waited for (bounded) before the CTA leaves, so no
  // copy into this CTA's shared memory is still in flight when it exits.
  int issued = 0, consumed = 0;
  const int polls = A.wait_polls;
  auto issue_chunk = [&](int c) {
    issued = c + 1;
    if (c == A.skip_chunk) return;  // failure-detection test: leave this chunk unissued
    const int x = a + c * T, xe = imin(x + T, e);
    const uint32_t sk = smem_addr(stages + (c % S) * STAGE);
    issue_rows<KT, VT, D>(A, kb, vb, x, xe, hlo, hhi, hk, hv, sk, sk + T * KROW, bar0 + 8 * (c % S));
  };

  const bool halo_issued = clustered && has_halo;
  if (tid == 0) {
    if (halo_issued) {  // hhi - hlo <= drop <= kClusterHaloRows rows (host-checked)
      const uint32_t n = uint32_t(hhi - hlo);
      mbar_arrive_expect_tx(halo_bar, n * (KROW + VROW));
      bulk_g2s(smem_addr(halo_sk), kb + size_t(hlo) * D, n * KROW, halo_bar);
      bulk_g2s(smem_addr(halo_sv), vb + size_t(hlo) * D, n * VROW, halo_bar);
    }
    const int pro = imin(S - 1, nchunks);
    for (int c = 0; c < pro; ++c) issue_chunk(c);
  }

  // The rotation table and the group's queries (plain loads) are requested while the
  // first chunks' copies are in flight, before any barrier.
  Lanes L;
  L.init(A);
  L.begin_pair(A, b, h);
  const uint8_t* mrow = A.mask != nullptr ? A.mask + b * A.mask_sb : nullptr;

  bool failed = false, halo_landed = !halo_issued;
  if (clustered) {
    // Every CTA of the cluster holds its halo rows before any CTA stores: a split reads the
    // first rows of the next split before that split overwrites them.  A CTA arrives once
    // its halo rows have landed and waits for the others' arrivals only before its first
    // store (after the first chunk's work), so the barrier's latency overlaps that work.
    if (halo_issued) {
      halo_landed = mbar_wait_bounded(halo_bar, 0, polls);
      if (!halo_landed) failed = true;
    }
    cluster_arrive();
  }

#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % S;
    if (!failed) {
      if (mbar_wait_bounded(bar0 + 8 * stage, (c / S) & 1, polls))
        consumed = c + 1;
      else
        failed = true;
    }
    const int x = a + c * T, xe = imin(x + T, e);
    KT* sk = reinterpret_cast<KT*>(stages + stage * STAGE);
    VT* sv = reinterpret_cast<VT*>(stages + stage * STAGE + T * KROW);
    if (A.append_row >= x && A.append_row < xe) {  // CTA-uniform
      fill_append_row<KT, VT, D, NT>(A, b, h, sk, sv, A.append_row - x);
      __syncthreads();
    }
    if (clustered && has_halo) {  // output rows whose sources are the staged halo rows
      const int r0 = imax(x, hlo - A.drop), r1 = imin(xe, hhi - A.drop);
      if (r0 < r1) {  // CTA-uniform
        copy_rows<KROW, VROW, NT>(reinterpret_cast<unsigned char*>(sk) + (r0 - x) * KROW,
                              reinterpret_cast<unsigned char*>(sv) + (r0 - x) * VROW,
                              halo_sk + (r0 + A.drop - hlo) * KROW, halo_sv + (r0 + A.drop - hlo) * VROW,
                              r1 - r0);
        __syncthreads();
      }
    }
    if (!failed) L.chunk(sk, sv, x, xe, A, mrow, kmir);
    int st_lo, st_hi;
    store_range(A, x, xe, st_lo, st_hi);
    fence_proxy_async_smem();
    failed = __syncthreads_or(failed);
    if (clustered && c == 0) cluster_wait();  // every halo of the cluster has landed
    if (tid == 0) {
      if (!failed && st_lo < st_hi) {
        bulk_s2g(kb + size_t(st_lo) * D, smem_addr(sk) + (st_lo - x) * KROW, uint32_t(st_hi - st_lo) * KROW);
        bulk_s2g(vb + size_t(st_lo) * D, smem_addr(sv) + (st_lo - x) * VROW, uint32_t(st_hi - st_lo) * VROW);
      }
      bulk_commit();
      const int nxt = c + S - 1;
      if (nxt < nchunks && !failed) {
        bulk_wait_read<1>();  // the store of chunk c-1 (same stage) has read its smem
        issue_chunk(nxt);
      }
    }
  }
  // The stores have read their shared memory (their global writes complete with the grid).
  if (tid == 0) bulk_wait_read<0>();
  failed = __syncthreads_or(failed);
  allow_dependents();
  if (failed && tid == 0) {
    atomicOr(A.status, 1);
    // Drain: every load issued but not seen to land (the chunk whose wait ran out included,
    // unless it was never issued) gets one more bounded wait.  At most S - 1 chunks are in
    // flight at a failure, on distinct stages, so each stage's phase is unambiguous.
    for (int c = consumed; c < issued; ++c)
      if (c != A.skip_chunk) mbar_wait_bounded(bar0 + 8 * (c % S), (c / S) & 1, polls);
    if (!halo_landed) mbar_wait_bounded(halo_bar, 0, polls);
  }
  // A clustered CTA stays for the cluster barriers below (its results are void).
  if (failed && !clustered) return;

  if constexpr (ATTEND) {
    float* scratch = reinterpret_cast<float*>(stages);
    L.to_scratch(scratch);
    __syncthreads();
    const int G = A.group;
    if (!clustered) {
      for (int idx = tid; idx < G * D; idx += NT) {
        const int g = idx / D, d = idx - g * D;
        float M, Ls, O;
        Lanes::from_scratch(scratch, g, d, M, Ls, O);
        if (A.ns == 1) {
          VT* o = reinterpret_cast<VT*>(A.out) + b * A.o_sb + (h * G + g) * A.o_sh;
          o[d] = Elem<VT>::from_f(O / Ls);
        } else {
          const size_t part = (size_t(p) * A.ns + j) * G + g;
          A.o_part[part * D + d] = O;
          if (d == 0) {
            A.m_part[part] = M;
            A.l_part[part] = Ls;
          }
        }
      }
      return;
    }
    // Clustered: the pair's G * D outputs are cut into ns equal slices, slice r merged by
    // the CTA of rank r.  Every CTA pushes each output of its partial into the owning CTA's
    // merge area (remote stores, no round trip) and its (M, L) per group into every CTA's;
    // after one cluster barrier each CTA merges its slice from its own shared memory.
    const int ns = A.ns;
    const int per = (G * D + ns - 1) / ns;
    float* recv_o = reinterpret_cast<float*>(halo_sv + kClusterHaloRows * VROW);  // [ns][per]
    float* recv_m = recv_o + GMAX * D + kClusterMax;                            // [GMAX][kClusterMax]
    float* recv_l = recv_m + GMAX * kClusterMax;
    float* wts = recv_l + GMAX * kClusterMax;
    const uint32_t o_addr = smem_addr(recv_o), m_addr = smem_addr(recv_m), l_addr = smem_addr(recv_l);
    for (int idx = tid; idx < G * D; idx += NT) {
      const int g = idx / D, d = idx - g * D;
      float M, Ls, O;
      Lanes::from_scratch(scratch, g, d, M, Ls, O);
      const int owner = idx / per;
      st_cluster_f32(cluster_map(o_addr + 4u * uint32_t(j * per + idx - owner * per), uint32_t(owner)), O);
      if (d == 0) {
        for (int r = 0; r < ns; ++r) {
          st_cluster_f32(cluster_map(m_addr + 4u * uint32_t(g * kClusterMax + j), uint32_t(r)), M);
          st_cluster_f32(cluster_map(l_addr + 4u * uint32_t(g * kClusterMax + j), uint32_t(r)), Ls);
        }
      }
    }
    cluster_sync();  // every push has landed; after this no CTA touches another's memory
    if (!failed) {   // CTA-uniform
      // normalised weights: one warp per group, one split per lane
      const int lane = tid & 31;
      for (int g = tid >> 5; g < G; g += NW) {
        const bool live = lane < ns;
        const float w = split_weight(live ? recv_m[g * kClusterMax + lane] : kNegInf,
                                     live ? recv_l[g * kClusterMax + lane] : 0.f);
        if (live) wts[g * kClusterMax + lane] = w;
      }
      __syncthreads();
      const int lo = j * per, hi = imin(lo + per, G * D);
      for (int idx = lo + tid; idx < hi; idx += NT) {
        const int g = idx / D, d = idx - g * D, i = idx - lo;
        float o = 0.f;
        for (int r = 0; r < ns; ++r) o = __fmaf_rn(wts[g * kClusterMax + r], recv_o[r * per + i], o);
        VT* op = reinterpret_cast<VT*>(A.out) + b * A.o_sb + (h * G + g) * A.o_sh;
        op[d] = Elem<VT>::from_f(o);
      }
    }
  }
}

// Byte geometry of the cache buffers for the type-agnostic halo copy.
struct HaloBytes {
  int64_t k_sb, k_sh, v_sb, v_sh;  // byte strides of batch / head
  int krow, vrow;                  // bytes per row (multiples of 16)
};

// 16-byte words of halo rows each thread of sink_halo_kernel copies per round (all loads of a
// round are issued before its stores).
constexpr int kHaloWordsPerThread = 4;

// Copies the halo rows of every split but the last into the workspace (pre-pass of an
// in-place shift that spans several splits).  Grid: (ceil(words / (kThreads *
// kHaloWordsPerThread)), batch * heads_kv), words = (ns - 1) * halo_rows * (K + V row words).
// A round of a thread covers words i, i + kThreads, ... of its CTA's tile, so every load
// instruction is coalesced and a round's loads are all in flight before the first store.
__global__ void __launch_bounds__(kThreads) sink_halo_kernel(const __grid_constant__ StreamArgs A,
                                                             const HaloBytes H) {
  allow_dependents();  // the stream kernel may launch; it waits for this grid to complete
  const int p = blockIdx.y;
  const int b = p / A.heads_kv, h = p - b * A.heads_kv;
  const int kv4 = H.krow / (int)sizeof(uint4), vv4 = H.vrow / (int)sizeof(uint4);
  const uint4* kbase = reinterpret_cast<const uint4*>(A.kbuf + b * H.k_sb + h * H.k_sh);
  const uint4* vbase = reinterpret_cast<const uint4*>(A.vbuf + b * H.v_sb + h * H.v_sh);
  // one flat index space over (split, halo row, 16-byte word), K words then V words
  const int nb = A.ns - 1;
  const int kper = A.halo_rows * kv4, vper = A.halo_rows * vv4;
  const int nk = nb * kper, total = nk + nb * vper;
  constexpr int U = kHaloWordsPerThread;
  for (int tile = blockIdx.x * (kThreads * U); tile < total; tile += gridDim.x * (kThreads * U)) {
    uint4 w[U];
    size_t dst[U];
    int kind[U];  // 0: nothing, 1: K word, 2: V word
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = tile + u * kThreads + threadIdx.x;
      kind[u] = 0;
      if (i >= total) continue;
      const bool isk = i < nk;
      const int per = isk ? kper : vper, w4 = isk ? kv4 : vv4;
      const int li = isk ? i : i - nk;
      const int j = li / per, r = (li % per) / w4, c = li % w4;
      int a, e;
      split_rows(A.row_begin, A.row_end, A.rows_per_split, j, a, e);
      int hlo, hhi;
      halo_range(A.n_sink, A.window, A.drop, A.written_end, false, a, e, hlo, hhi);
      if (hlo + r >= hhi) continue;
      dst[u] = ((size_t(p) * A.ns + j) * A.halo_rows + r) * w4 + c;
      w[u] = isk ? kbase[size_t(hlo + r) * kv4 + c] : vbase[size_t(hlo + r) * vv4 + c];
      kind[u] = isk ? 1 : 2;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (kind[u] == 1) reinterpret_cast<uint4*>(A.halo_k)[dst[u]] = w[u];
      else if (kind[u] == 2) reinterpret_cast<uint4*>(A.halo_v)[dst[u]] = w[u];
    }
  }
}

// Log-sum-exp merge of the ns split partials of every (batch, kv-head) pair.  Grid
// (pairs, G * D / 32): a CTA merges 32 consecutive outputs of one query row g (D is a
// multiple of 32).  Warp 0 turns the ns (max, sum) pairs of row g into normalised weights;
// then, with more than 32 splits, the 4 warps each sum every 4th split's partial (lane =
// output, coalesced) and the 4 sums are added in warp order; with at most 32 splits warp 0
// sums them all in split order.  Either way the result does not depend on scheduling.
template <typename VT, int D>
__global__ void __launch_bounds__(kThreads) sink_combine_kernel(const float* __restrict__ o_part,
                                                                const float* __restrict__ m_part,
                                                                const float* __restrict__ l_part,
                                                                char* out, int64_t o_sb,
                                                                int64_t o_sh, int heads_kv, int G,
                                                                int ns) {
  __shared__ float wts[kMaxSplits];
  __shared__ float sums[kWarps][32];
  grid_dependency_wait();  // the partials of the stream kernel are complete
  const int p = blockIdx.x;
  const int b = p / heads_kv, h = p - b * heads_kv;
  const int first = blockIdx.y * 32;  // first output (g * D + d) of this CTA
  const int g = first / D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t base = size_t(p) * ns;
  if (warp == 0) {
    float mx = kNegInf;
    for (int s = lane; s < ns; s += 32) mx = fmaxf(mx, m_part[(base + s) * G + g]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
    const float mref = mx == kNegInf ? 0.f : mx;
    float sum = 0.f;
    for (int s = lane; s < ns; s += 32)
      sum = __fmaf_rn(exp2f(m_part[(base + s) * G + g] - mref), l_part[(base + s) * G + g], sum);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off);
    const float inv = 1.f / sum;
    for (int s = lane; s < ns; s += 32) wts[s] = exp2f(m_part[(base + s) * G + g] - mref) * inv;
  }
  __syncthreads();
  const int d = first - g * D + lane;
  const int nsub = ns > 32 ? kWarps : 1;
  if (warp < nsub) {
    float o = 0.f;
    for (int s = warp; s < ns; s += nsub) o = __fmaf_rn(wts[s], o_part[((base + s) * G + g) * D + d], o);
    sums[warp][lane] = o;
  }
  __syncthreads();
  if (warp == 0) {
    float o = sums[0][lane];
    for (int w = 1; w < nsub; ++w) o += sums[w][lane];
    VT* op = reinterpret_cast<VT*>(out) + b * o_sb + (h * G + g) * o_sh;
    op[d] = Elem<VT>::from_f(o);
  }
}

// kbuf[:, :, row + t] = k_new[:, :, t] (converted), vbuf likewise, for t < n.
template <typename KT, typename VT>
__global__ void sink_append_kernel(KT* kbuf, VT* vbuf, int64_t k_sb, int64_t k_sh, int64_t v_sb,
                                   int64_t v_sh, const VT* knew, const VT* vnew, int64_t kn_sb,
                                   int64_t kn_sh, int64_t kn_st, int64_t vn_sb, int64_t vn_sh,
                                   int64_t vn_st, int heads, int n, int D, int row, int64_t total) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int d = int(i % D);
    int64_t r = i / D;
    const int t = int(r % n);
    r /= n;
    const int h = int(r % heads);
    const int b = int(r / heads);
    const VT kx = knew[b * kn_sb + h * kn_sh + t * kn_st + d];
    const VT vx = vnew[b * vn_sb + h * vn_sh + t * vn_st + d];
    kbuf[b * k_sb + h * k_sh + int64_t(row + t) * D + d] = Elem<KT>::from_f(Elem<VT>::to_f(kx));
    vbuf[b * v_sb + h * v_sh + int64_t(row + t) * D + d] = vx;
  }
}

}  // namespace sinkb200
