// Ring-buffer ("v2") cache step: the new token is written over one ring slot and the few
// region keys (sinks, pinned tokens) are rotated from their stored originals to sit just
// before the window (src/sinkcache/cache_v2.py:101-116 _rotate_region, :167-181
// _decode_step).  Window keys are never touched; attention over ring + region runs on the
// tensor-core kernel (sink_attend_tc_kernel) for 16-bit keys at head_dim 128, else on the
// stream kernel in attend-only mode, then the split combine.
#pragma once

#include "sink_common.cuh"

namespace sinkb200 {

struct V2PlaceArgs {
  char* kbuf;                        // ring + region slots, rows contiguous
  char* vbuf;
  int64_t k_sb, k_sh, v_sb, v_sh;    // element strides
  const char* knew;                  // [B, Hkv, 1, D] new token, or null (no ring write)
  const char* vnew;
  int64_t kn_sb, kn_sh, vn_sb, vn_sh;
  const char* reg_k;                 // [B, Hkv, >= R, D] region keys at their original rotation
  int64_t rk_sb, rk_sh, rk_st;
  char* rout;                        // [B, Hkv, >= R, D] rotated region keys
  int64_t ro_sb, ro_sh, ro_st;
  const int64_t* reg_pos;            // [>= R] original positions of the region tokens
  int64_t* position;                 // {t, arrivals} on the device, or null: t_host
  int64_t t_host;
  const double* inv_freq;            // [rot_half]
  int n_sink, window, ring, R, rot_half, heads_kv, pairs;
};

// First window position when the next token is t.
__device__ __forceinline__ long long v2_window_start(const V2PlaceArgs& a, long long t) {
  long long ws = t < a.n_sink ? t : a.n_sink;
  if (t - a.window > ws) ws = t - a.window;
  return ws;
}

// The place work of one (batch, kv-head) pair, limited to its rows [row_lo, row_hi) of the
// kv buffers (ring slots, then the region rows from `ring`): the new token into ring slot
// (t - n_sink) mod ring when that slot is in range, and the region rows j (kv row ring + j,
// or region_out row j) in range rotated from their originals.  Region row j is rotated by
// (ws - R + j) - reg_pos[j]; the angle is formed in fp64 (positions grow without bound),
// cos/sin rounded once to fp32, and each output element is fp32(fp32(x * cos) +
// fp32(rotate_half(x) * sin)) rounded once to the storage type: the reference's three
// separately rounded tensor ops.  Threads `tid` of `nthreads` share the work.
template <typename T, int D>
__device__ __forceinline__ void v2_place_pair(const V2PlaceArgs& a, int b, int h, long long t, long long ws,
                                              int row_lo, int row_hi, int tid, int nthreads) {
  using E = Elem<T>;
  constexpr int kVec = 16 / sizeof(T);   // elements per 16-byte vector
  constexpr int kRowVecs = D / kVec;
  if (a.knew) {
    long long slot = (t - a.n_sink) % a.ring;
    if (slot < 0) slot += a.ring;
    if (slot >= row_lo && slot < row_hi) {
      for (int i = tid; i < 2 * kRowVecs; i += nthreads) {
        const bool is_v = i >= kRowVecs;
        const int c = is_v ? i - kRowVecs : i;
        const T* src = reinterpret_cast<const T*>(is_v ? a.vnew : a.knew) +
                       (is_v ? b * a.vn_sb + h * a.vn_sh : b * a.kn_sb + h * a.kn_sh);
        T* dst = reinterpret_cast<T*>(is_v ? a.vbuf : a.kbuf) +
                 (is_v ? b * a.v_sb + h * a.v_sh : b * a.k_sb + h * a.k_sh) + slot * D;
        reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
      }
    }
  }
  const int j0 = row_lo - a.ring > 0 ? row_lo - a.ring : 0;
  const int j1 = row_hi - a.ring < a.R ? row_hi - a.ring : a.R;
  if (j0 >= j1) return;
  const T* rk = reinterpret_cast<const T*>(a.reg_k) + b * a.rk_sb + h * a.rk_sh;
  T* ro = reinterpret_cast<T*>(a.rout) + b * a.ro_sb + h * a.ro_sh;
  const int rh = a.rot_half, pass = D - 2 * rh;
  const int per_row = rh + pass;
  for (int i = tid; i < (j1 - j0) * per_row; i += nthreads) {
    const int j = j0 + i / per_row, c = i % per_row;
    const T* x = rk + j * a.rk_st;
    T* y = ro + j * a.ro_st;
    if (c < rh) {
      const long long delta = ws - a.R + j - a.reg_pos[j];
      const double ang = __dmul_rn(static_cast<double>(delta), a.inv_freq[c]);
      double sd, cd;
      sincos(ang, &sd, &cd);  // one argument reduction for both
      const float cs = __double2float_rn(cd);
      const float sn = __double2float_rn(sd);
      const float x1 = E::to_f(x[c]), x2 = E::to_f(x[c + rh]);
      y[c] = E::from_f(__fadd_rn(__fmul_rn(x1, cs), __fmul_rn(-x2, sn)));
      y[c + rh] = E::from_f(__fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn)));
    } else {
      const int d = 2 * rh + (c - rh);
      y[d] = x[d];
    }
  }
}

// Counts this CTA in on the device position after it has read t: the last CTA of the grid to
// arrive stores t + 1 and clears the counter (no CTA waits for another).
__device__ __forceinline__ void v2_position_arrive(const V2PlaceArgs& a, long long t) {
  __threadfence();
  const unsigned long long prev = atomicAdd(reinterpret_cast<unsigned long long*>(a.position + 1), 1ull);
  if (prev == gridDim.x - 1) {
    a.position[0] = t + 1;
    a.position[1] = 0;
    __threadfence();
  }
}

// One CTA per (batch, kv-head) pair (grid-strided): the whole place step of each pair (the new
// token, every region row).  With `position`, the last CTA to finish stores t + 1.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) sink_v2_place_kernel(V2PlaceArgs a) {
  grid_dependency_wait();
  allow_dependents();
  __shared__ long long t_s;
  if (threadIdx.x == 0) t_s = a.position ? a.position[0] : a.t_host;
  __syncthreads();
  const long long t = t_s;
  const long long ws = v2_window_start(a, t);
  for (int p = blockIdx.x; p < a.pairs; p += gridDim.x) {
    const int b = p / a.heads_kv, h = p - b * a.heads_kv;
    v2_place_pair<T, D>(a, b, h, t, ws, 0, a.ring + a.R, threadIdx.x, kThreads);
  }
  if (a.position) {
    __syncthreads();
    if (threadIdx.x == 0) v2_position_arrive(a, t);
  }
}

}  // namespace sinkb200

namespace sinkb200 {

// Rows a ring-buffer layer's multi-token step attends over, in the reference's order:
// [region (R rows), window by position, chunk (n rows)].
struct V2GatherArgs {
  const char* kbuf;                  // ring + region slots, rows contiguous
  const char* vbuf;
  int64_t k_sb, k_sh, v_sb, v_sh;    // element strides
  const char* knew;                  // [B, Hkv, n, D] the chunk, or null (n == 0)
  const char* vnew;
  int64_t kn_sb, kn_sh, kn_st, vn_sb, vn_sh, vn_st;
  char* ok;                          // [B, Hkv, >= rows, D] outputs
  char* ov;
  int64_t ok_sb, ok_sh, ok_st, ov_sb, ov_sh, ov_st;
  int64_t lo;                        // first window position (>= n_sink)
  int n_sink, ring, R, nwin, n, rows, heads_kv, pairs;
};

// 16-byte words each thread of sink_v2_gather_kernel copies per round (loads before stores).
constexpr int kGatherWordsPerThread = 4;

// out rows r of every (batch, head): r < R: the region's value row (kv row ring + r; the
// region's keys are rotated into out_k by the place kernel); R <= r < R + nwin: ring slot
// (lo + r - R - n_sink) mod ring; then chunk row r - R - nwin.  One flat index over
// (tensor, pair, row, 16-byte word), consecutive threads on consecutive words of a row.
template <typename T, int D>
__global__ void __launch_bounds__(kThreads) sink_v2_gather_kernel(const __grid_constant__ V2GatherArgs g) {
  grid_dependency_wait();
  allow_dependents();
  constexpr int W = D * int(sizeof(T)) / 16;  // words per row
  const long long per = (long long)g.pairs * g.rows * W;
  const long long total = 2 * per;
  constexpr int U = kGatherWordsPerThread;
  const long long step = (long long)gridDim.x * kThreads * U;
  for (long long tile = (long long)blockIdx.x * kThreads * U; tile < total; tile += step) {
    uint4 w[U];
    uint4* dst[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long long i = tile + (long long)u * kThreads + threadIdx.x;
      dst[u] = nullptr;
      if (i >= total) continue;
      const bool isv = i >= per;
      const long long li = isv ? i - per : i;
      const int c = int(li % W);
      const long long rr = li / W;
      const int r = int(rr % g.rows), p = int(rr / g.rows);
      const int b = p / g.heads_kv, h = p - b * g.heads_kv;
      const T* src;
      if (r < g.R) {
        if (!isv) continue;
        src = reinterpret_cast<const T*>(g.vbuf) + b * g.v_sb + h * g.v_sh + (long long)(g.ring + r) * D;
      } else if (r < g.R + g.nwin) {
        long long slot = (g.lo + (r - g.R) - g.n_sink) % g.ring;
        if (slot < 0) slot += g.ring;
        src = isv ? reinterpret_cast<const T*>(g.vbuf) + b * g.v_sb + h * g.v_sh + slot * D
                  : reinterpret_cast<const T*>(g.kbuf) + b * g.k_sb + h * g.k_sh + slot * D;
      } else {
        const int j = r - g.R - g.nwin;
        src = isv ? reinterpret_cast<const T*>(g.vnew) + b * g.vn_sb + h * g.vn_sh + (long long)j * g.vn_st
                  : reinterpret_cast<const T*>(g.knew) + b * g.kn_sb + h * g.kn_sh + (long long)j * g.kn_st;
      }
      T* d = isv ? reinterpret_cast<T*>(g.ov) + b * g.ov_sb + h * g.ov_sh + (long long)r * g.ov_st
                 : reinterpret_cast<T*>(g.ok) + b * g.ok_sb + h * g.ok_sh + (long long)r * g.ok_st;
      w[u] = reinterpret_cast<const uint4*>(src)[c];
      dst[u] = reinterpret_cast<uint4*>(d) + c;
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (dst[u] != nullptr) *dst[u] = w[u];
  }
}

}  // namespace sinkb200
