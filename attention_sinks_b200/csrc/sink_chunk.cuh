// Per-lane state and per-chunk work shared by the stream kernels: re-rotation of window
// keys, q.k scores for a GQA group, online softmax and P.V over one shared-memory chunk,
// and the merge of a CTA's four warps.
//
// Lane layout (StreamGeom): LPR lanes share one cache row; lane i of a row owns K dims
// [4i, 4i+4) and their RoPE partners [D/2 + 4i, D/2 + 4i + 4), and V dims [8i, 8i + 8).
// A warp covers RPW rows per step; a chunk of T rows is STEPS steps of all warps.
#pragma once

#include "sink_common.cuh"

namespace sinkb200 {

constexpr uint32_t kFull = 0xffffffffu;
constexpr float kNegInf = -__builtin_inff();

// Normalised softmax weight of split `lane` of one query row in a merge of ns <= 32 split
// partials, one split per lane (lanes >= ns pass m = -inf, l = 0): exp2(m - max) divided by
// sum over splits of exp2(m_s - max) * l_s.  The maximum and the sum are reduced over the
// whole warp in the same butterfly order as sink_combine_kernel, so an in-cluster merge gets
// the same weights as the combine launch.
__device__ __forceinline__ float split_weight(float m, float l) {
  float mx = m;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, off));
  const float mref = mx == kNegInf ? 0.f : mx;
  const float e = exp2f(m - mref);
  float sum = __fmaf_rn(e, l, 0.f);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) sum += __shfl_xor_sync(kFull, sum, off);
  return e * (1.f / sum);
}

// NW warps per CTA share each chunk: warp w takes row groups w, w + NW, ... (T / (NW * RPW)
// steps of RPW rows).  The chunk geometry (T rows) does not depend on NW.
template <typename KT, typename VT, int D, int GMAX, bool ATTEND, int NW = kWarps>
struct StreamLanes {
  using Gm = StreamGeom<KT, VT, D>;
  static constexpr int LPR = Gm::LPR, RPW = Gm::RPW;
  static constexpr int STEPS = Gm::T / (NW * RPW);
  static_assert(STEPS * NW * RPW == Gm::T && STEPS >= 1, "warps per chunk");
  static constexpr int NG = ATTEND ? GMAX : 1;

  int warp, lane, li, rg;
  bool rotating;
  float cs[4], sn[4];
  float qlo[NG][4], qhi[NG][4];
  float m[NG], l[NG], acc[NG][8];

  __device__ __forceinline__ void init(const StreamArgs& A) {
    warp = threadIdx.x >> 5;
    lane = threadIdx.x & 31;
    li = lane % LPR;
    rg = lane / LPR;
    rotating = A.drop > 0 && A.rotate != 0;
    if (rotating) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        cs[i] = A.cos_tab[4 * li + i];
        sn[i] = A.sin_tab[4 * li + i];
      }
    }
  }

  // Start a new (batch, kv-head) pair: zero the softmax state, load the group's queries
  // pre-scaled by scale * log2(e).
  __device__ __forceinline__ void begin_pair(const StreamArgs& A, int b, int h) {
    reset_softmax();
    load_queries(A, b, h);
  }

  // Zero the online-softmax state (a new item of the same pair).
  __device__ __forceinline__ void reset_softmax() {
    if constexpr (ATTEND) {
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
        m[g] = kNegInf;
        l[g] = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[g][k] = 0.f;
      }
    }
  }

  __device__ __forceinline__ void load_queries(const StreamArgs& A, int b, int h) {
    if constexpr (ATTEND) {
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
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
  }

  // One chunk of rows [x, xe) staged at sk / sv (row t of the chunk at sk + t * D):
  // window rows are re-rotated in place in shared memory, then (ATTEND) scored and folded
  // into the online softmax.  `mrow`: optional per-row mask of this pair.  `mirror`
  // (optional): this pair's key copy in the value type; row r of it gets row r's key.
  __device__ __forceinline__ void chunk(KT* sk, const VT* sv, int x, int xe, const StreamArgs& A,
                                        const uint8_t* mrow, VT* mirror = nullptr) {
    const int wend = A.n_sink + A.window;
    float sc[NG][STEPS];
#pragma unroll
    for (int i = 0; i < STEPS; ++i) {
      const int t = i * (NW * RPW) + warp * RPW + rg;
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
      if (mirror != nullptr && valid) {  // the row's final key, in the value type
        VT* mrow_k = mirror + size_t(r) * D;
        Elem<VT>::store4(mrow_k + 4 * li, lo);
        Elem<VT>::store4(mrow_k + D / 2 + 4 * li, hi);
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
          sc[g][i] = seen ? d : kNegInf;
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
        const float mref = mnew == kNegInf ? 0.f : mnew;
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
        const int t = i * (NW * RPW) + warp * RPW + rg;
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
  }

  // Scratch floats the warp merge needs.
  static constexpr int kScratchFloats = NW * GMAX * (D + 2);

  // Reduce the row groups of each warp and write (m, l, acc) of every warp to `scratch`.
  // The caller synchronises the CTA before reading the scratch back.
  __device__ __forceinline__ void to_scratch(float* scratch) {
    if constexpr (ATTEND) {
#pragma unroll
      for (int g = 0; g < GMAX; ++g) {
#pragma unroll
        for (int off = LPR; off < 32; off <<= 1) {
          l[g] += __shfl_xor_sync(kFull, l[g], off);
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[g][k] += __shfl_xor_sync(kFull, acc[g][k], off);
        }
      }
      float* sm_m = scratch;
      float* sm_l = sm_m + NW * GMAX;
      float* sm_acc = sm_l + NW * GMAX;
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
    }
  }

  // The CTA's (M, L, O) for entry (g, d) from the warps' scratch (log2-domain max M,
  // normaliser L, unnormalised output O).
  static __device__ __forceinline__ void from_scratch(const float* scratch, int g, int d, float& M,
                                                      float& L, float& O) {
    const float* sm_m = scratch;
    const float* sm_l = sm_m + NW * GMAX;
    const float* sm_acc = sm_l + NW * GMAX;
    M = kNegInf;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, sm_m[w * GMAX + g]);
    const float Mref = M == kNegInf ? 0.f : M;
    L = 0.f;
    O = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float wt = exp2f(sm_m[w * GMAX + g] - Mref);
      L = __fmaf_rn(wt, sm_l[w * GMAX + g], L);
      O = __fmaf_rn(wt, sm_acc[(w * GMAX + g) * D + d], O);
    }
  }
};

}  // namespace sinkb200
