// Kernels of the sink-cache decode path.
//
//   sink_stream_kernel  one pass over the cache rows of a (batch, kv-head, split) work item:
//                       bulk-copy (TMA) row chunks into a shared-memory pipeline, re-rotate
//                       window keys in fp32 registers, write shifted rows back with bulk
//                       stores, and (ATTEND) run an online-softmax GQA decode attention over
//                       the same rows.  With drop == 0 and no append row it is a plain
//                       split-K decode attention; with ATTEND == false a plain eviction.
//   sink_halo_kernel    copies the few source rows that a later split overwrites before an
//                       earlier split reads them (in-place shift across split boundaries).
//   sink_combine_kernel merges the per-split softmax partials (log-sum-exp weights).
//   sink_append_kernel  writes new K/V rows (unfused path).
#pragma once

#include "sink_common.cuh"

namespace sinkb200 {

constexpr uint32_t kFull = 0xffffffffu;

template <typename KT, typename VT, int D, int GMAX, bool ATTEND>
__global__ void __launch_bounds__(kThreads) sink_stream_kernel(const __grid_constant__ StreamArgs A) {
  using Gm = StreamGeom<KT, VT, D>;
  constexpr int LPR = Gm::LPR, RPW = Gm::RPW, T = Gm::T, S = Gm::S, STEPS = Gm::STEPS;
  constexpr int KROW = Gm::KROW, VROW = Gm::VROW, STAGE = Gm::STAGE;
  constexpr float NEG_INF = -__builtin_inff();

  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t bar0 = smem_addr(smem);
  unsigned char* stages = smem + kBarrierBytes;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int li = lane % LPR;  // lane within its row
  const int rg = lane / LPR;  // row group within the warp
  const int j = blockIdx.x, p = blockIdx.y;
  const int b = p / A.heads_kv, h = p - b * A.heads_kv;

  int a, e;
  split_rows(A.row_begin, A.row_end, A.rows_per_split, j, a, e);
  int hlo, hhi;
  halo_range(A.n_sink, A.window, A.drop, A.written_end, A.ns, j, a, e, hlo, hhi);
  const bool has_halo = hlo < hhi;

  KT* kb = reinterpret_cast<KT*>(A.kbuf) + b * A.k_sb + h * A.k_sh;
  VT* vb = reinterpret_cast<VT*>(A.vbuf) + b * A.v_sb + h * A.v_sh;
  const size_t halo_row0 = (size_t(p) * A.ns + j) * A.halo_rows;
  const KT* hk = reinterpret_cast<const KT*>(A.halo_k) + halo_row0 * D;
  const VT* hv = reinterpret_cast<const VT*>(A.halo_v) + halo_row0 * D;
  const int nchunks = (e - a + T - 1) / T;
  const int wend = A.n_sink + A.window;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // One thread issues every bulk copy of chunk c: up to four contiguous source segments
  // (unshifted rows, shifted rows read directly, shifted rows from the halo, shifted rows
  // read directly above the rows this launch writes).  The append row comes from threads.
  auto issue_chunk = [&](int c) {
    const int stage = c % S;
    const int x = a + c * T, xe = imin(x + T, e);
    const uint32_t sk = smem_addr(stages + stage * STAGE);
    const uint32_t sv = sk + T * KROW;
    const uint32_t bar = bar0 + 8 * stage;
    int seg_t[4], seg_n[4];
    const KT* seg_k[4];
    const VT* seg_v[4];
    int nseg = 0;
    const int lowlim = A.drop > 0 ? A.n_sink : (A.append_row >= 0 ? A.append_row : A.row_end);
    const int p1 = imin(xe, lowlim);
    if (x < p1) {
      seg_t[nseg] = 0;
      seg_n[nseg] = p1 - x;
      seg_k[nseg] = kb + size_t(x) * D;
      seg_v[nseg] = vb + size_t(x) * D;
      ++nseg;
    }
    if (A.drop > 0) {
      const int w0 = imax(x, A.n_sink), w1 = imin(xe, wend);
      if (w0 < w1) {
        const int s0 = w0 + A.drop, s1 = w1 + A.drop;
        const int d1 = has_halo ? imin(s1, hlo) : s1;
        if (s0 < d1) {
          seg_t[nseg] = s0 - A.drop - x;
          seg_n[nseg] = d1 - s0;
          seg_k[nseg] = kb + size_t(s0) * D;
          seg_v[nseg] = vb + size_t(s0) * D;
          ++nseg;
        }
        if (has_halo) {
          const int h0 = imax(s0, hlo), h1 = imin(s1, hhi);
          if (h0 < h1) {
            seg_t[nseg] = h0 - A.drop - x;
            seg_n[nseg] = h1 - h0;
            seg_k[nseg] = hk + size_t(h0 - hlo) * D;
            seg_v[nseg] = hv + size_t(h0 - hlo) * D;
            ++nseg;
          }
          const int u0 = imax(s0, hhi);
          if (u0 < s1) {
            seg_t[nseg] = u0 - A.drop - x;
            seg_n[nseg] = s1 - u0;
            seg_k[nseg] = kb + size_t(u0) * D;
            seg_v[nseg] = vb + size_t(u0) * D;
            ++nseg;
          }
        }
      }
    }
    uint32_t bytes = 0;
    for (int i = 0; i < nseg; ++i) bytes += uint32_t(seg_n[i]) * (KROW + VROW);
    mbar_arrive_expect_tx(bar, bytes);
    for (int i = 0; i < nseg; ++i) {
      bulk_g2s(sk + seg_t[i] * KROW, seg_k[i], uint32_t(seg_n[i]) * KROW, bar);
      bulk_g2s(sv + seg_t[i] * VROW, seg_v[i], uint32_t(seg_n[i]) * VROW, bar);
    }
  };

  if (tid == 0) {
    const int pro = imin(S - 1, nchunks);
    for (int c = 0; c < pro; ++c) issue_chunk(c);
  }

  // Lane constants: the rotation for angle -drop (first half of the HF table; both halves
  // are equal) and the group's queries pre-scaled by scale * log2(e).
  float cs[4], sn[4];
  const bool rotating = A.drop > 0 && A.rotate != 0;
  if (rotating) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      cs[i] = A.cos_tab[4 * li + i];
      sn[i] = A.sin_tab[4 * li + i];
    }
  }
  const uint8_t* mrow = A.mask != nullptr ? A.mask + b * A.mask_sb : nullptr;
  float qlo[ATTEND ? GMAX : 1][4], qhi[ATTEND ? GMAX : 1][4];
  float m[ATTEND ? GMAX : 1], l[ATTEND ? GMAX : 1], acc[ATTEND ? GMAX : 1][8];
  if constexpr (ATTEND) {
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
      m[g] = NEG_INF;
      l[g] = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[g][k] = 0.f;
      if (g < A.group) {
        const VT* qp = reinterpret_cast<const VT*>(A.q) + b * A.q_sb + (h * A.group + g) * A.q_sh;
        float t4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) t4[i] = Elem<VT>::to_f(qp[4 * li + i]);
#pragma unroll
        for (int i = 0; i < 4; ++i) qlo[g][i] = t4[i] * A.scale_log2;
#pragma unroll
        for (int i = 0; i < 4; ++i) t4[i] = Elem<VT>::to_f(qp[D / 2 + 4 * li + i]);
#pragma unroll
        for (int i = 0; i < 4; ++i) qhi[g][i] = t4[i] * A.scale_log2;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) qlo[g][i] = qhi[g][i] = 0.f;
      }
    }
  }

  bool failed = false;
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % S;
    if (!mbar_wait_bounded(bar0 + 8 * stage, (c / S) & 1)) failed = true;
    const int x = a + c * T, xe = imin(x + T, e);
    KT* sk = reinterpret_cast<KT*>(stages + stage * STAGE);
    VT* sv = reinterpret_cast<VT*>(stages + stage * STAGE + T * KROW);

    if (A.append_row >= x && A.append_row < xe) {  // CTA-uniform
      const int t = A.append_row - x;
      const VT* kn = reinterpret_cast<const VT*>(A.knew) + b * A.kn_sb + h * A.kn_sh;
      const VT* vn = reinterpret_cast<const VT*>(A.vnew) + b * A.vn_sb + h * A.vn_sh;
      for (int d = tid; d < D; d += kThreads) {
        sk[t * D + d] = Elem<KT>::from_f(Elem<VT>::to_f(kn[d]));
        sv[t * D + d] = vn[d];
      }
      __syncthreads();
    }

    float sc[ATTEND ? GMAX : 1][STEPS];
#pragma unroll
    for (int i = 0; i < STEPS; ++i) {
      const int t = i * (kWarps * RPW) + warp * RPW + rg;
      const int r = x + t;
      const bool valid = r < xe;
      float lo[4], hi[4];
      KT* krow = sk + t * D;
      Elem<KT>::load4(krow + 4 * li, lo);
      Elem<KT>::load4(krow + D / 2 + 4 * li, hi);
      if (rotating && valid && r >= A.n_sink && r < wend) {
        // rope(x, -drop) in the order SinkLayer._rerotate evaluates it:
        // x * cos + roll(x, D/2) * sin_signed, with the product-add fused (one rounding).
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float y1 = __fmaf_rn(hi[k], -sn[k], __fmul_rn(lo[k], cs[k]));
          const float y2 = __fmaf_rn(lo[k], sn[k], __fmul_rn(hi[k], cs[k]));
          lo[k] = Elem<KT>::round(y1);
          hi[k] = Elem<KT>::round(y2);
        }
        Elem<KT>::store4(krow + 4 * li, lo);
        Elem<KT>::store4(krow + D / 2 + 4 * li, hi);
      }
      if constexpr (ATTEND) {
        const bool seen = valid && (mrow == nullptr || mrow[r] != 0);
#pragma unroll
        for (int g = 0; g < GMAX; ++g) {
          float d = 0.f;
#pragma unroll
          for (int k = 0; k < 4; ++k) d = __fmaf_rn(qlo[g][k], lo[k], d);
#pragma unroll
          for (int k = 0; k < 4; ++k) d = __fmaf_rn(qhi[g][k], hi[k], d);
#pragma unroll
          for (int off = LPR / 2; off >= 1; off >>= 1) d += __shfl_xor_sync(kFull, d, off);
          sc[g][i] = seen ? d : NEG_INF;
        }
      }
    }

    if constexpr (ATTEND) {
      // online softmax over this chunk's rows of the warp (m is warp-uniform)
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        float mx = sc[g][0];
#pragma unroll
        for (int i = 1; i < STEPS; ++i) mx = fmaxf(mx, sc[g][i]);
#pragma unroll
        for (int off = LPR; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
        const float mnew = fmaxf(m[g], mx);
        const float mref = mnew == NEG_INF ? 0.f : mnew;
        if (mnew > m[g]) {
          const float alpha = exp2f(m[g] - mref);
          l[g] *= alpha;
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[g][k] *= alpha;
          m[g] = mnew;
        }
#pragma unroll
        for (int i = 0; i < STEPS; ++i) {
          sc[g][i] = exp2f(sc[g][i] - mref);
          l[g] += sc[g][i];
        }
      }
#pragma unroll
      for (int i = 0; i < STEPS; ++i) {
        const int t = i * (kWarps * RPW) + warp * RPW + rg;
        if (x + t < xe) {
          float v[8];
          Elem<VT>::load8(sv + t * D + 8 * li, v);
#pragma unroll
          for (int g = 0; g < GMAX; ++g) {
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[g][k] = __fmaf_rn(sc[g][i], v[k], acc[g][k]);
          }
        }
      }
    }

    // rows this chunk writes back: window rows (drop > 0) and the append row
    int st_lo = 0, st_hi = 0;
    if (A.drop > 0) {
      st_lo = imax(x, A.n_sink);
      st_hi = imin(xe, wend + (A.append_row >= 0 ? 1 : 0));
    } else if (A.append_row >= 0) {
      st_lo = imax(x, A.append_row);
      st_hi = imin(xe, A.append_row + 1);
    }
    fence_proxy_async_smem();
    failed = __syncthreads_or(failed);
    if (failed) break;
    if (tid == 0) {
      if (st_lo < st_hi) {
        const uint32_t src_k = smem_addr(sk) + (st_lo - x) * KROW;
        const uint32_t src_v = smem_addr(sv) + (st_lo - x) * VROW;
        bulk_s2g(kb + size_t(st_lo) * D, src_k, uint32_t(st_hi - st_lo) * KROW);
        bulk_s2g(vb + size_t(st_lo) * D, src_v, uint32_t(st_hi - st_lo) * VROW);
      }
      bulk_commit();
      const int nxt = c + S - 1;
      if (nxt < nchunks) {
        bulk_wait_read<1>();  // the store of chunk c-1 (same stage) has read its smem
        issue_chunk(nxt);
      }
    }
  }
  if (tid == 0) bulk_wait<0>();
  __syncthreads();
  if (failed) {
    if (tid == 0) atomicOr(A.status, 1);
    return;
  }

  if constexpr (ATTEND) {
    // merge the row groups of each warp, then the 4 warps, through shared memory
#pragma unroll
    for (int g = 0; g < GMAX; ++g) {
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1) {
        l[g] += __shfl_xor_sync(kFull, l[g], off);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[g][k] += __shfl_xor_sync(kFull, acc[g][k], off);
      }
    }
    float* sm_m = reinterpret_cast<float*>(stages);
    float* sm_l = sm_m + kWarps * GMAX;
    float* sm_acc = sm_l + kWarps * GMAX;
    if (lane < LPR) {
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
#pragma unroll
        for (int k = 0; k < 8; ++k) sm_acc[(warp * GMAX + g) * D + 8 * lane + k] = acc[g][k];
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        sm_m[warp * GMAX + g] = m[g];
        sm_l[warp * GMAX + g] = l[g];
      }
    }
    __syncthreads();
    const int G = A.group;
    for (int idx = tid; idx < G * D; idx += kThreads) {
      const int g = idx / D, d = idx - g * D;
      float M = NEG_INF;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm_m[w * GMAX + g]);
      const float Mref = M == NEG_INF ? 0.f : M;
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float wt = exp2f(sm_m[w * GMAX + g] - Mref);
        L = __fmaf_rn(wt, sm_l[w * GMAX + g], L);
        O = __fmaf_rn(wt, sm_acc[(w * GMAX + g) * D + d], O);
      }
      if (A.ns == 1) {
        VT* o = reinterpret_cast<VT*>(A.out) + b * A.o_sb + (h * G + g) * A.o_sh;
        o[d] = Elem<VT>::from_f(O / L);
      } else {
        const size_t part = (size_t(p) * A.ns + j) * G + g;
        A.o_part[part * D + d] = O;
        if (d == 0) {
          A.m_part[part] = M;
          A.l_part[part] = L;
        }
      }
    }
  }
}

// Byte geometry of the cache buffers for the type-agnostic halo copy.
struct HaloBytes {
  int64_t k_sb, k_sh, v_sb, v_sh;  // byte strides of batch / head
  int krow, vrow;                  // bytes per row (multiples of 16)
};

// Copies the halo rows of every split but the last into the workspace (pre-pass of an
// in-place shift that spans several splits).
__global__ void __launch_bounds__(kThreads) sink_halo_kernel(const __grid_constant__ StreamArgs A,
                                                             const HaloBytes H) {
  const int j = blockIdx.x, p = blockIdx.y;
  const int b = p / A.heads_kv, h = p - b * A.heads_kv;
  int a, e;
  split_rows(A.row_begin, A.row_end, A.rows_per_split, j, a, e);
  int hlo, hhi;
  halo_range(A.n_sink, A.window, A.drop, A.written_end, A.ns, j, a, e, hlo, hhi);
  if (hlo >= hhi) return;
  const size_t halo_row0 = (size_t(p) * A.ns + j) * A.halo_rows;
  const int kv4 = H.krow / (int)sizeof(uint4), vv4 = H.vrow / (int)sizeof(uint4);
  const uint4* ks = reinterpret_cast<const uint4*>(A.kbuf + b * H.k_sb + h * H.k_sh) + size_t(hlo) * kv4;
  const uint4* vs = reinterpret_cast<const uint4*>(A.vbuf + b * H.v_sb + h * H.v_sh) + size_t(hlo) * vv4;
  uint4* kd = reinterpret_cast<uint4*>(A.halo_k) + halo_row0 * kv4;
  uint4* vd = reinterpret_cast<uint4*>(A.halo_v) + halo_row0 * vv4;
  const int nk = (hhi - hlo) * kv4, nv = (hhi - hlo) * vv4;
  for (int i = threadIdx.x; i < nk; i += kThreads) kd[i] = ks[i];
  for (int i = threadIdx.x; i < nv; i += kThreads) vd[i] = vs[i];
}

// Log-sum-exp merge of the ns split partials of every (batch, kv-head) pair.
template <typename VT, int D>
__global__ void __launch_bounds__(kThreads) sink_combine_kernel(const float* __restrict__ o_part,
                                                                const float* __restrict__ m_part,
                                                                const float* __restrict__ l_part,
                                                                char* out, int64_t o_sb,
                                                                int64_t o_sh, int heads_kv, int G,
                                                                int ns) {
  __shared__ float wts[kMaxSplits * kMaxGroup];
  const int p = blockIdx.x;
  const int b = p / heads_kv, h = p - b * heads_kv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t base = size_t(p) * ns;
  for (int g = warp; g < G; g += kWarps) {
    float mx = -__builtin_inff();
    for (int s = lane; s < ns; s += 32) mx = fmaxf(mx, m_part[(base + s) * G + g]);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
    const float mref = mx == -__builtin_inff() ? 0.f : mx;
    float sum = 0.f;
    for (int s = lane; s < ns; s += 32)
      sum = __fmaf_rn(exp2f(m_part[(base + s) * G + g] - mref), l_part[(base + s) * G + g], sum);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off);
    const float inv = 1.f / sum;
    for (int s = lane; s < ns; s += 32)
      wts[s * G + g] = exp2f(m_part[(base + s) * G + g] - mref) * inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int g = idx / D, d = idx - g * D;
    float o = 0.f;
    for (int s = 0; s < ns; ++s) o = __fmaf_rn(wts[s * G + g], o_part[((base + s) * G + g) * D + d], o);
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
