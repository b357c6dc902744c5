// C ABI of the sink-cache decode path (include/sinkcache_b200.h): argument checks, the
// split plan, workspace layout and kernel dispatch over (K type, V type, head_dim, group).
#include <atomic>
#include <climits>
#include <cstring>

#include "../../include/sinkcache_b200.h"
#include "sink_kernels.cuh"

using namespace sinkb200;

namespace {

int elem_size(int32_t dt) {
  switch (dt) {
    case SINK_DTYPE_F32: return 4;
    case SINK_DTYPE_BF16: return 2;
    case SINK_DTYPE_F16: return 2;
    default: return 0;
  }
}

// (K storage, model dtype) pairs with kernels: fp32 or model-dtype keys, V in the model dtype.
bool supported_types(int32_t kdt, int32_t vdt) {
  if (vdt == SINK_DTYPE_BF16) return kdt == SINK_DTYPE_F32 || kdt == SINK_DTYPE_BF16;
  if (vdt == SINK_DTYPE_F16) return kdt == SINK_DTYPE_F32 || kdt == SINK_DTYPE_F16;
  if (vdt == SINK_DTYPE_F32) return kdt == SINK_DTYPE_F32;
  return false;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct Plan {
  int T = 0, S = 0, stage = 0, smem = 0, ctas_per_sm = 0;
  int ns = 1, rows_per_split = 0, halo_rows = 0;
  size_t off_o = 0, off_m = 0, off_l = 0, off_hk = 0, off_hv = 0, total = 256;
};

// Must agree with StreamGeom<KT, VT, D> (checked again at launch).
bool geometry(int D, int ks, int vs, Plan& pl) {
  if (D != 64 && D != 128 && D != 256) return false;
  const int lpr = D / 8, rpw = 32 / lpr;
  pl.T = 4 * kWarps * rpw;
  pl.stage = pl.T * D * (ks + vs);
  int s = kPipeBytes / pl.stage;
  pl.S = s < 2 ? 2 : (s > 4 ? 4 : s);
  pl.smem = kBarrierBytes + pl.S * pl.stage;
  pl.ctas_per_sm = kSmemPerSM / (pl.smem + kSmemReservedPerCTA);
  if (pl.ctas_per_sm < 1) pl.ctas_per_sm = 1;
  return true;
}

// Split plan: every (batch, head) pair's rows cut into `ns` items of `tps` chunks, one CTA
// each.  Two regimes, from measurements over the op-bench grid on B200:
//   - a step whose pairs fit in one wave of CTAs with items of at most kMaxItemChunks
//     chunks takes exactly one wave: as many splits per pair as there are free SM slots
//     per pair (few pairs with long rows: every SM streams one long item);
//   - otherwise items of kMinItemChunks..kMaxItemChunks chunks, aiming at kTargetWaves
//     waves, so the block scheduler evens out SMs that stream at different rates.
constexpr long kMinItemChunks = 4;
constexpr long kMaxItemChunks = 32;
constexpr long kTargetWaves = 16;

void choose_splits(int pairs, int rows, int T, int slots, Plan& pl) {
  const long tiles = (rows + T - 1) / T;
  const long total = long(pairs) * tiles;
  long ns;
  if (long(pairs) * ((tiles + kMaxItemChunks - 1) / kMaxItemChunks) <= slots) {
    ns = slots / pairs;
  } else {
    long tps = (total + kTargetWaves * slots - 1) / (kTargetWaves * slots);
    tps = tps < kMinItemChunks ? kMinItemChunks : (tps > kMaxItemChunks ? kMaxItemChunks : tps);
    ns = (tiles + tps - 1) / tps;
  }
  if (ns > tiles) ns = tiles;
  if (ns > kMaxSplits) ns = kMaxSplits;
  if (ns < 1) ns = 1;
  const long tps = (tiles + ns - 1) / ns;  // even the items out
  pl.ns = int((tiles + tps - 1) / tps);
  pl.rows_per_split = int(tps) * T;
}

int32_t make_plan(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q, int32_t D,
                  int32_t kdt, int32_t vdt, int32_t rows, int32_t n_sink, int32_t window,
                  int32_t drop, int32_t num_sms, Plan& pl) {
  pl = Plan();
  if (batch < 1 || heads_kv < 1 || num_sms < 1 || num_sms > 4096) return SINK_EINVAL;
  if (long(batch) * heads_kv > (1L << 24)) return SINK_EINVAL;  // pair indices stay in int
  if (!supported_types(kdt, vdt)) return SINK_EDTYPE;
  const int ks = elem_size(kdt), vs = elem_size(vdt);
  if (!geometry(D, ks, vs, pl)) return SINK_EHEADDIM;
  if (op == SINK_OP_APPEND) return SINK_OK;
  const bool attend = op == SINK_OP_ATTEND || op == SINK_OP_FUSED_STEP;
  int G = 1;
  if (attend) {
    if (heads_q < heads_kv || heads_q % heads_kv) return SINK_EGROUP;
    G = heads_q / heads_kv;
    if (G > kMaxGroup) return SINK_EGROUP;
  }
  if (n_sink < 0 || window < 1 || drop < 0) return SINK_EINVAL;
  int nrows;
  if (op == SINK_OP_EVICT) nrows = window;
  else if (op == SINK_OP_ATTEND || op == SINK_OP_FUSED_STEP) nrows = rows;
  else return SINK_EINVAL;
  if (nrows < 1) return SINK_EINVAL;
  const int pairs = batch * heads_kv;
  choose_splits(pairs, nrows, pl.T, num_sms * pl.ctas_per_sm, pl);
  size_t off = 256;  // status word
  if (attend && pl.ns > 1) {
    const size_t parts = size_t(pairs) * pl.ns * G;
    pl.off_o = off;
    off += align256(parts * D * 4);
    pl.off_m = off;
    off += align256(parts * 4);
    pl.off_l = off;
    off += align256(parts * 4);
  }
  const bool evicts = op == SINK_OP_EVICT || op == SINK_OP_FUSED_STEP;
  if (evicts && drop > 0 && pl.ns > 1) {
    pl.halo_rows = drop < pl.rows_per_split ? drop : pl.rows_per_split;
    const size_t hrows = size_t(pairs) * pl.ns * pl.halo_rows;
    pl.off_hk = off;
    off += align256(hrows * D * ks);
    pl.off_hv = off;
    off += align256(hrows * D * vs);
  }
  pl.total = off;
  return SINK_OK;
}

int device_sms(int* dev_out) {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  *dev_out = dev;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int32_t check_kv(const sink_kv_buffers_t* kv) {
  if (!kv || !kv->k || !kv->v) return SINK_EINVAL;
  if (kv->batch < 1 || kv->heads_kv < 1 || kv->slots < 1) return SINK_EINVAL;
  if (!supported_types(kv->k_dtype, kv->v_dtype)) return SINK_EDTYPE;
  const int D = kv->head_dim;
  if (D != 64 && D != 128 && D != 256) return SINK_EHEADDIM;
  const int ks = elem_size(kv->k_dtype), vs = elem_size(kv->v_dtype);
  // bulk copies need 16-byte aligned row starts for every (batch, head)
  if (!aligned16(kv->k) || !aligned16(kv->v)) return SINK_ELAYOUT;
  if (((kv->k_stride_b * ks) & 15) || ((kv->k_stride_h * ks) & 15)) return SINK_ELAYOUT;
  if (((kv->v_stride_b * vs) & 15) || ((kv->v_stride_h * vs) & 15)) return SINK_ELAYOUT;
  if (kv->k_stride_b < 0 || kv->k_stride_h < 0 || kv->v_stride_b < 0 || kv->v_stride_h < 0)
    return SINK_ELAYOUT;
  return SINK_OK;
}

int32_t check_rows(const sink_rows_t* r, int32_t dtype, int32_t batch, int32_t heads, int32_t n) {
  if (!r || !r->data) return SINK_EINVAL;
  if (r->dtype != dtype) return SINK_EDTYPE;
  if (r->heads != heads || r->n != n) return SINK_EINVAL;
  (void)batch;
  return SINK_OK;
}

template <typename KT, typename VT, int D, int GMAX, bool ATTEND>
int32_t launch_stream(const StreamArgs& A, const Plan& pl, int pairs, cudaStream_t st, int dev) {
  using Gm = StreamGeom<KT, VT, D>;
  if (Gm::SMEM != pl.smem || Gm::T != pl.T) return SINK_EINVAL;  // host/device geometry drift
  auto kern = sink_stream_kernel<KT, VT, D, GMAX, ATTEND>;
  static std::atomic<uint64_t> configured{0};
  const uint64_t bit = uint64_t(1) << dev;
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::SMEM);
    if (err != cudaSuccess) return err;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  kern<<<dim3(pl.ns, pairs), kThreads, Gm::SMEM, st>>>(A);
  return cudaGetLastError();
}

template <bool ATTEND, typename KT, typename VT, int D>
int32_t by_group(int G, const StreamArgs& A, const Plan& pl, int pairs, cudaStream_t st, int dev) {
  if constexpr (!ATTEND) {
    (void)G;
    return launch_stream<KT, VT, D, 1, false>(A, pl, pairs, st, dev);
  } else {
    if (G <= 1) return launch_stream<KT, VT, D, 1, true>(A, pl, pairs, st, dev);
    if (G <= 2) return launch_stream<KT, VT, D, 2, true>(A, pl, pairs, st, dev);
    if (G <= 4) return launch_stream<KT, VT, D, 4, true>(A, pl, pairs, st, dev);
    return launch_stream<KT, VT, D, 8, true>(A, pl, pairs, st, dev);
  }
}

template <bool ATTEND, typename KT, typename VT>
int32_t by_dim(int D, int G, const StreamArgs& A, const Plan& pl, int pairs, cudaStream_t st, int dev) {
  switch (D) {
    case 64: return by_group<ATTEND, KT, VT, 64>(G, A, pl, pairs, st, dev);
    case 128: return by_group<ATTEND, KT, VT, 128>(G, A, pl, pairs, st, dev);
    case 256: return by_group<ATTEND, KT, VT, 256>(G, A, pl, pairs, st, dev);
    default: return SINK_EHEADDIM;
  }
}

template <bool ATTEND>
int32_t dispatch_stream(int kdt, int vdt, int D, int G, const StreamArgs& A, const Plan& pl,
                        int pairs, cudaStream_t st, int dev) {
  if (vdt == SINK_DTYPE_BF16) {
    if (kdt == SINK_DTYPE_F32) return by_dim<ATTEND, float, __nv_bfloat16>(D, G, A, pl, pairs, st, dev);
    if (kdt == SINK_DTYPE_BF16) return by_dim<ATTEND, __nv_bfloat16, __nv_bfloat16>(D, G, A, pl, pairs, st, dev);
  } else if (vdt == SINK_DTYPE_F16) {
    if (kdt == SINK_DTYPE_F32) return by_dim<ATTEND, float, __half>(D, G, A, pl, pairs, st, dev);
    if (kdt == SINK_DTYPE_F16) return by_dim<ATTEND, __half, __half>(D, G, A, pl, pairs, st, dev);
  } else if (vdt == SINK_DTYPE_F32) {
    if (kdt == SINK_DTYPE_F32) return by_dim<ATTEND, float, float>(D, G, A, pl, pairs, st, dev);
  }
  return SINK_EDTYPE;
}

template <typename VT>
int32_t launch_combine_t(int D, const StreamArgs& A, int pairs, cudaStream_t st) {
  switch (D) {
    case 64:
      sink_combine_kernel<VT, 64><<<pairs, kThreads, 0, st>>>(A.o_part, A.m_part, A.l_part, A.out, A.o_sb, A.o_sh, A.heads_kv, A.group, A.ns);
      break;
    case 128:
      sink_combine_kernel<VT, 128><<<pairs, kThreads, 0, st>>>(A.o_part, A.m_part, A.l_part, A.out, A.o_sb, A.o_sh, A.heads_kv, A.group, A.ns);
      break;
    case 256:
      sink_combine_kernel<VT, 256><<<pairs, kThreads, 0, st>>>(A.o_part, A.m_part, A.l_part, A.out, A.o_sb, A.o_sh, A.heads_kv, A.group, A.ns);
      break;
    default: return SINK_EHEADDIM;
  }
  return cudaGetLastError();
}

int32_t launch_combine(int vdt, int D, const StreamArgs& A, int pairs, cudaStream_t st) {
  if (vdt == SINK_DTYPE_BF16) return launch_combine_t<__nv_bfloat16>(D, A, pairs, st);
  if (vdt == SINK_DTYPE_F16) return launch_combine_t<__half>(D, A, pairs, st);
  if (vdt == SINK_DTYPE_F32) return launch_combine_t<float>(D, A, pairs, st);
  return SINK_EDTYPE;
}

int32_t launch_halo(const sink_kv_buffers_t* kv, const StreamArgs& A, const Plan& pl, int pairs,
                    cudaStream_t st) {
  if (pl.ns < 2 || A.drop <= 0) return SINK_OK;
  HaloBytes H;
  const int ks = elem_size(kv->k_dtype), vs = elem_size(kv->v_dtype);
  H.k_sb = kv->k_stride_b * ks;
  H.k_sh = kv->k_stride_h * ks;
  H.v_sb = kv->v_stride_b * vs;
  H.v_sh = kv->v_stride_h * vs;
  H.krow = kv->head_dim * ks;
  H.vrow = kv->head_dim * vs;
  sink_halo_kernel<<<dim3(pl.ns - 1, pairs), kThreads, 0, st>>>(A, H);
  return cudaGetLastError();
}

void fill_common(StreamArgs& A, const sink_kv_buffers_t* kv, const Plan& pl, char* ws) {
  std::memset(&A, 0, sizeof(A));
  A.kbuf = static_cast<char*>(kv->k);
  A.vbuf = static_cast<char*>(kv->v);
  A.k_sb = kv->k_stride_b;
  A.k_sh = kv->k_stride_h;
  A.v_sb = kv->v_stride_b;
  A.v_sh = kv->v_stride_h;
  A.heads_kv = kv->heads_kv;
  A.group = 1;
  A.append_row = -1;
  A.ns = pl.ns;
  A.rows_per_split = pl.rows_per_split;
  A.halo_rows = pl.halo_rows;
  A.status = reinterpret_cast<int*>(ws);
  A.o_part = pl.off_o ? reinterpret_cast<float*>(ws + pl.off_o) : nullptr;
  A.m_part = pl.off_m ? reinterpret_cast<float*>(ws + pl.off_m) : nullptr;
  A.l_part = pl.off_l ? reinterpret_cast<float*>(ws + pl.off_l) : nullptr;
  A.halo_k = pl.off_hk ? ws + pl.off_hk : nullptr;
  A.halo_v = pl.off_hv ? ws + pl.off_hv : nullptr;
}

constexpr float kLog2e = 1.4426950408889634f;

template <typename KT, typename VT>
int32_t launch_append_t(const sink_kv_buffers_t* kv, const sink_rows_t* kn, const sink_rows_t* vn,
                        int32_t row, cudaStream_t st) {
  const int64_t total = int64_t(kv->batch) * kv->heads_kv * kn->n * kv->head_dim;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  sink_append_kernel<KT, VT><<<int(blocks), threads, 0, st>>>(
      static_cast<KT*>(kv->k), static_cast<VT*>(kv->v), kv->k_stride_b, kv->k_stride_h,
      kv->v_stride_b, kv->v_stride_h, static_cast<const VT*>(kn->data),
      static_cast<const VT*>(vn->data), kn->stride_b, kn->stride_h, kn->stride_t, vn->stride_b,
      vn->stride_h, vn->stride_t, kv->heads_kv, kn->n, kv->head_dim, row, total);
  return cudaGetLastError();
}

}  // namespace

extern "C" {

int32_t sink_abi_version(void) { return SINK_ABI_VERSION; }

const char* sink_strerror(int32_t code) {
  switch (code) {
    case SINK_OK: return "ok";
    case SINK_EINVAL: return "sinkcache_b200: size or index out of range";
    case SINK_EDTYPE: return "sinkcache_b200: unsupported dtype combination (K fp32 or model dtype; V, q, new rows in the model dtype bf16/fp16/fp32)";
    case SINK_EHEADDIM: return "sinkcache_b200: head_dim must be 64, 128 or 256";
    case SINK_EGROUP: return "sinkcache_b200: heads_q / heads_kv must be an integer between 1 and 8";
    case SINK_ELAYOUT: return "sinkcache_b200: cache rows must be contiguous and 16-byte aligned";
    case SINK_EWORKSPACE: return "sinkcache_b200: workspace missing or smaller than sink_workspace_bytes()";
    case SINK_EDEVICE: return "sinkcache_b200: no usable CUDA device";
    case SINK_ESCRATCH: return "sinkcache_b200: request needs more than the 16 MiB static scratch of sink_decode_attention_noalloc; use sink_decode_attention with a workspace";
    default:
      if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
      return "sinkcache_b200: unknown error";
  }
}

size_t sink_workspace_bytes(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q,
                            int32_t head_dim, int32_t k_dtype, int32_t v_dtype, int32_t rows,
                            int32_t n_sink, int32_t window, int32_t drop, int32_t num_sms) {
  Plan pl;
  if (make_plan(op, batch, heads_kv, heads_q, head_dim, k_dtype, v_dtype, rows, n_sink, window,
                drop, num_sms, pl) != SINK_OK)
    return 0;
  return pl.total;
}

int32_t sink_plan(int32_t op, int32_t batch, int32_t heads_kv, int32_t heads_q, int32_t head_dim,
                  int32_t k_dtype, int32_t v_dtype, int32_t rows, int32_t n_sink, int32_t window,
                  int32_t drop, int32_t num_sms, int32_t* splits, int32_t* rows_per_split,
                  int32_t* chunk_rows, int32_t* stages, int32_t* smem_bytes) {
  Plan pl;
  const int32_t rc = make_plan(op, batch, heads_kv, heads_q, head_dim, k_dtype, v_dtype, rows,
                               n_sink, window, drop, num_sms, pl);
  if (rc != SINK_OK) return rc;
  if (splits) *splits = pl.ns;
  if (rows_per_split) *rows_per_split = pl.rows_per_split;
  if (chunk_rows) *chunk_rows = pl.T;
  if (stages) *stages = pl.S;
  if (smem_bytes) *smem_bytes = pl.smem;
  return SINK_OK;
}

int32_t sink_append(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                    const sink_rows_t* v_new, int32_t row, void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if ((rc = check_rows(k_new, kv->v_dtype, kv->batch, kv->heads_kv, k_new ? k_new->n : 0))) return rc;
  if ((rc = check_rows(v_new, kv->v_dtype, kv->batch, kv->heads_kv, k_new->n))) return rc;
  if (k_new->n < 1 || row < 0 || row + k_new->n > kv->slots) return SINK_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int kdt = kv->k_dtype, vdt = kv->v_dtype;
  if (vdt == SINK_DTYPE_BF16) {
    if (kdt == SINK_DTYPE_F32) return launch_append_t<float, __nv_bfloat16>(kv, k_new, v_new, row, st);
    return launch_append_t<__nv_bfloat16, __nv_bfloat16>(kv, k_new, v_new, row, st);
  }
  if (vdt == SINK_DTYPE_F16) {
    if (kdt == SINK_DTYPE_F32) return launch_append_t<float, __half>(kv, k_new, v_new, row, st);
    return launch_append_t<__half, __half>(kv, k_new, v_new, row, st);
  }
  return launch_append_t<float, float>(kv, k_new, v_new, row, st);
}

int32_t sink_evict_rerotate(const sink_kv_buffers_t* kv, int32_t n_sink, int32_t window,
                            int32_t drop, const float* cos_tab, const float* sin_tab,
                            int32_t rotate, void* workspace, size_t workspace_bytes,
                            void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if (n_sink < 0 || window < 1 || drop < 0) return SINK_EINVAL;
  if (int64_t(n_sink) + window + drop > kv->slots) return SINK_EINVAL;
  if (drop == 0) return SINK_OK;
  if (rotate && (!cos_tab || !sin_tab)) return SINK_EINVAL;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  Plan pl;
  rc = make_plan(SINK_OP_EVICT, kv->batch, kv->heads_kv, kv->heads_kv, kv->head_dim, kv->k_dtype,
                 kv->v_dtype, 0, n_sink, window, drop, sms, pl);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.total || !aligned16(workspace)) return SINK_EWORKSPACE;
  StreamArgs A;
  fill_common(A, kv, pl, static_cast<char*>(workspace));
  A.n_sink = n_sink;
  A.window = window;
  A.drop = drop;
  A.rotate = rotate ? 1 : 0;
  A.cos_tab = cos_tab;
  A.sin_tab = sin_tab;
  A.row_begin = n_sink;
  A.row_end = n_sink + window;
  A.written_end = n_sink + window;
  const int pairs = kv->batch * kv->heads_kv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = launch_halo(kv, A, pl, pairs, st))) return rc;
  return dispatch_stream<false>(kv->k_dtype, kv->v_dtype, kv->head_dim, 1, A, pl, pairs, st, dev);
}

int32_t sink_decode_attention(const sink_rows_t* q, const sink_kv_buffers_t* kv, int32_t rows,
                              float scale, const uint8_t* mask, int64_t mask_stride_b,
                              void* out, int64_t out_stride_b, int64_t out_stride_h,
                              void* workspace, size_t workspace_bytes, void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if (!q || !q->data || !out) return SINK_EINVAL;
  if (q->dtype != kv->v_dtype) return SINK_EDTYPE;
  if (q->n != 1 || rows < 1 || rows > kv->slots) return SINK_EINVAL;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  Plan pl;
  rc = make_plan(SINK_OP_ATTEND, kv->batch, kv->heads_kv, q->heads, kv->head_dim, kv->k_dtype,
                 kv->v_dtype, rows, 0, 1, 0, sms, pl);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.total || !aligned16(workspace)) return SINK_EWORKSPACE;
  StreamArgs A;
  fill_common(A, kv, pl, static_cast<char*>(workspace));
  A.group = q->heads / kv->heads_kv;
  A.q = static_cast<const char*>(q->data);
  A.q_sb = q->stride_b;
  A.q_sh = q->stride_h;
  A.out = static_cast<char*>(out);
  A.o_sb = out_stride_b;
  A.o_sh = out_stride_h;
  A.window = 1;
  A.row_begin = 0;
  A.row_end = rows;
  A.written_end = 0;
  A.scale_log2 = scale * kLog2e;
  A.mask = mask;
  A.mask_sb = mask_stride_b;
  const int pairs = kv->batch * kv->heads_kv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = dispatch_stream<true>(kv->k_dtype, kv->v_dtype, kv->head_dim, A.group, A, pl, pairs, st, dev)))
    return rc;
  if (pl.ns > 1) return launch_combine(kv->v_dtype, kv->head_dim, A, pairs, st);
  return SINK_OK;
}

int32_t sink_fused_decode_step(const sink_kv_buffers_t* kv, const sink_rows_t* k_new,
                               const sink_rows_t* v_new, const sink_rows_t* q,
                               int32_t n_sink, int32_t window, int32_t drop,
                               int32_t append_row, const float* cos_tab, const float* sin_tab,
                               int32_t rotate, float scale, const uint8_t* mask,
                               int64_t mask_stride_b, void* out, int64_t out_stride_b,
                               int64_t out_stride_h, void* workspace, size_t workspace_bytes,
                               void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if ((rc = check_rows(k_new, kv->v_dtype, kv->batch, kv->heads_kv, 1))) return rc;
  if ((rc = check_rows(v_new, kv->v_dtype, kv->batch, kv->heads_kv, 1))) return rc;
  if (!q || !q->data || !out) return SINK_EINVAL;
  if (q->dtype != kv->v_dtype) return SINK_EDTYPE;
  if (q->n != 1) return SINK_EINVAL;
  if (n_sink < 0 || window < 1 || drop < 0 || append_row < 0 || append_row >= kv->slots)
    return SINK_EINVAL;
  if (drop > 0) {
    if (append_row != n_sink + window) return SINK_EINVAL;
    if (int64_t(n_sink) + window + drop > kv->slots) return SINK_EINVAL;
    if (rotate && (!cos_tab || !sin_tab)) return SINK_EINVAL;
  }
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  Plan pl;
  rc = make_plan(SINK_OP_FUSED_STEP, kv->batch, kv->heads_kv, q->heads, kv->head_dim,
                 kv->k_dtype, kv->v_dtype, append_row + 1, n_sink, window, drop, sms, pl);
  if (rc) return rc;
  if (!workspace || workspace_bytes < pl.total || !aligned16(workspace)) return SINK_EWORKSPACE;
  StreamArgs A;
  fill_common(A, kv, pl, static_cast<char*>(workspace));
  A.group = q->heads / kv->heads_kv;
  A.knew = static_cast<const char*>(k_new->data);
  A.vnew = static_cast<const char*>(v_new->data);
  A.kn_sb = k_new->stride_b;
  A.kn_sh = k_new->stride_h;
  A.vn_sb = v_new->stride_b;
  A.vn_sh = v_new->stride_h;
  A.q = static_cast<const char*>(q->data);
  A.q_sb = q->stride_b;
  A.q_sh = q->stride_h;
  A.out = static_cast<char*>(out);
  A.o_sb = out_stride_b;
  A.o_sh = out_stride_h;
  A.cos_tab = cos_tab;
  A.sin_tab = sin_tab;
  A.n_sink = n_sink;
  A.window = window;
  A.drop = drop;
  A.rotate = rotate ? 1 : 0;
  A.row_begin = 0;
  A.row_end = append_row + 1;
  A.append_row = append_row;
  A.written_end = drop > 0 ? n_sink + window + 1 : append_row + 1;
  A.scale_log2 = scale * kLog2e;
  A.mask = mask;
  A.mask_sb = mask_stride_b;
  const int pairs = kv->batch * kv->heads_kv;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = launch_halo(kv, A, pl, pairs, st))) return rc;
  if ((rc = dispatch_stream<true>(kv->k_dtype, kv->v_dtype, kv->head_dim, A.group, A, pl, pairs, st, dev)))
    return rc;
  if (pl.ns > 1) return launch_combine(kv->v_dtype, kv->head_dim, A, pairs, st);
  return SINK_OK;
}

int32_t sink_read_status(void* workspace, void* stream, int32_t* status) {
  if (!workspace || !status) return SINK_EINVAL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t host = 0;
  cudaError_t err = cudaMemcpyAsync(&host, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  if (err == cudaSuccess) err = cudaMemsetAsync(workspace, 0, sizeof(int32_t), st);
  if (err == cudaSuccess) err = cudaStreamSynchronize(st);
  *status = host;
  return err;
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation variant

// Scratch of sink_decode_attention_noalloc.  In host code this name is only a stand-in for
// the symbol, not a device address: the host looks up each device's copy with
// cudaGetSymbolAddress and passes that pointer to the kernels.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SINK_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of g_noalloc_scratch on device `dev` (the current device), looked up once.
int32_t noalloc_scratch(int dev, void** ptr) {
  static std::atomic<void*> cache[64];
  void* p = cache[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess) return err;
    if (p == nullptr) return SINK_EDEVICE;
    cache[dev].store(p, std::memory_order_release);
  }
  *ptr = p;
  return SINK_OK;
}

}  // namespace

extern "C" int32_t sink_decode_attention_noalloc(const sink_rows_t* q, const sink_kv_buffers_t* kv,
                                                 int32_t rows, float scale, const uint8_t* mask,
                                                 int64_t mask_stride_b, void* out,
                                                 int64_t out_stride_b, int64_t out_stride_h,
                                                 void* stream) {
  int32_t rc = check_kv(kv);
  if (rc) return rc;
  if (!q || !q->data || !out) return SINK_EINVAL;
  int dev = 0;
  const int sms = device_sms(&dev);
  if (sms <= 0) return SINK_EDEVICE;
  Plan pl;
  rc = make_plan(SINK_OP_ATTEND, kv->batch, kv->heads_kv, q->heads, kv->head_dim, kv->k_dtype,
                 kv->v_dtype, rows, 0, 1, 0, sms, pl);
  if (rc) return rc;
  if (pl.total > SINK_NOALLOC_SCRATCH_BYTES) return SINK_ESCRATCH;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(dev, &scratch))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t err = cudaMemsetAsync(scratch, 0, sizeof(int32_t), st);  // status word
  if (err != cudaSuccess) return err;
  return sink_decode_attention(q, kv, rows, scale, mask, mask_stride_b, out, out_stride_b,
                               out_stride_h, scratch, SINK_NOALLOC_SCRATCH_BYTES, stream);
}
